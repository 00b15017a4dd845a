"""Graph runners of the DeLS draft-scoring path on the B200 kernels (drop-in for the
reference's ``kernel`` package)."""
