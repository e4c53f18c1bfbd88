"""aiter.ops stand-in (only `shuffle`)."""
