"""oscar_b200.engine"""
