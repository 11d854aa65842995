"""octopus_b200.models"""
