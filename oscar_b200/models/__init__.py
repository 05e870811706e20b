"""oscar_b200.models"""
