"""oscar_b200.ops"""
