"""Torch-backed stand-in for the few Apple-MLX primitives that mlx-vision-mamba calls.

Fixture-generation infrastructure only (tests/golden/make_golden.py puts this
directory on sys.path so the reference's own Python source can be imported and
run on the CPU).  Each primitive follows MLX's documented semantics; arrays are
torch tensors, so torch autograd supplies the reference code's gradients.
Metal kernels (`mx.fast.metal_kernel`) cannot run and raise when called.
"""
