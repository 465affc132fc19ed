"""CPU oracle for the GPTQ W4A16 quantized linear.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this package.
Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` use it, and only as the checker / the timed CPU reference.
"""
