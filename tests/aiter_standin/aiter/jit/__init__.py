"""aiter.jit stand-in (only `utils.chip_info`)."""
