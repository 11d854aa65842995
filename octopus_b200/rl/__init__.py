"""octopus_b200.rl"""
