"""oscar_b200.kv"""
