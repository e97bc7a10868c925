"""Test package of the B200 backend (one module name per test file for cross-file helpers)."""
