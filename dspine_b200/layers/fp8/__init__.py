"""FP8 coarse retrieval + BF16 rescore (the reference's ``sglang_dspine.layers.fp8``)."""
