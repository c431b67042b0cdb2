"""Host modules at the reference's ``sglang_dspine.sampling.sparse`` paths."""
