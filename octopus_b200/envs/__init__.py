"""octopus_b200.envs"""
