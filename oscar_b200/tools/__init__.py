"""oscar_b200.tools"""
