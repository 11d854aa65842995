"""octopus_b200.serving"""
