"""Module-level switches read by the quantized linear, as in
After-Revision-DROFELL/operators/flags.py:6-11 (the subset this path reads)."""
RECONSTRUCTE_WEIGTH_FLOAT16 = False
RECONSTRUCTE_WEIGTH_BFLOAT16 = False
REUSE_RECONSTRUCT_CACHE_WHEN_GRAD = True
