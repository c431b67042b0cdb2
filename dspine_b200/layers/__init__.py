"""Host modules at the reference's ``sglang_dspine.layers`` paths."""
