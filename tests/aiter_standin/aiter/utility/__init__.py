"""aiter.utility stand-in (only `fp4_utils`)."""
