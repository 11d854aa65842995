"""octopus_b200.runtime"""
