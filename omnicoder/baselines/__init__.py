"""Comparison builds written with stock PyTorch only (no kernel of this package).

:mod:`omnicoder.baselines.torch_nccl` is the plain torch.distributed (NCCL) +
cuBLAS build of the MoE pretraining step that the benchmark compares against.
The reference project has no multi-GPU path of its own (its launcher,
src/omnicoder/tools/torchrun_ep.py:7-18, only initialises a process group), so
this baseline is written here, with the same model, data and optimiser.
"""
