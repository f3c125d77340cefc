"""Reference-arm benchmark harness (runs the unmodified reference installed in baseline/_ref)."""
