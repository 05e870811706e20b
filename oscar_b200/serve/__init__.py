"""oscar_b200.serve"""
