"""Host modules at the reference's ``sglang_dspine.verification`` paths."""
