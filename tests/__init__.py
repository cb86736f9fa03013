"""Test suite of the B200 StrideWeave carrier."""
