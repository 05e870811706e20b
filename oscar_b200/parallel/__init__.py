"""oscar_b200.parallel"""
