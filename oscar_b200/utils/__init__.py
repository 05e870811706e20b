"""oscar_b200.utils"""
