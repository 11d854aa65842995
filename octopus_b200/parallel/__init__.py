"""Multi-GPU plumbing: process groups, data parallelism, FSDP, tensor parallelism,
symmetric peer memory and the fused compute+collective kernels' host side."""
