"""CPU oracle for the selective-scan hot path of mlx-vision-mamba.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
directory; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg (and `bench.py --impl reference`) use it, as the checker / CPU baseline.

Contents
  scan_ref.py   : `selective_scan` (mamba_block.py:20-74) and
                  `selective_scan_chunked` (mamba_fast.py:17-75) restated in
                  torch with the reference's operation order; gradients come
                  from torch autograd.
  model_ref.py  : MambaBlock, Residual/Bidirectional/MultiDirectional blocks,
                  the permutation helpers, patch embeddings and VisionMamba
                  (mamba_block.py:77-566, vision_mamba.py:25-228, vit.py:48-92)
                  restated on the CPU, with the reference's permute -> flip ->
                  block -> flip -> unpermute data movement kept literally.

Pinning.  The reference cannot run here as shipped (it needs Apple MLX).  The
fixtures under tests/golden/ were produced by executing the reference's own
Python source (mlx_vision_mamba/*.py, imported read-only) on top of a small
torch-backed stand-in for the MLX primitives it calls (tests/golden/mlx_shim);
tests/test_oracle_golden.py checks this oracle against those fixtures.  The
Metal kernels themselves cannot run (no Metal on Linux/NVIDIA), so the
gradient formulas are pinned through autograd of the reference's sequential
code instead.
"""
