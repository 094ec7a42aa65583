"""Runtime: ctypes binding of the C ABI (_lib), torch-facing ops, encoder executor."""
