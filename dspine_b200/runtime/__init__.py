"""Host modules at the reference's ``sglang_dspine.runtime`` paths."""
