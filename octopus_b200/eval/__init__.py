"""octopus_b200.eval"""
