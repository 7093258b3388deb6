"""Test oracle for the NVFP4 path (TEST INFRASTRUCTURE; never on the product path)."""
