"""Software-engineering environment: git workspace with sandboxed tools, container
executors, the nokill guard, test-based rewards."""
