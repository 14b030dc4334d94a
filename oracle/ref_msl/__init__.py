"""Host build of the reference kernels (test infrastructure only)."""
