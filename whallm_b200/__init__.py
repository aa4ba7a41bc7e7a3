"""B200-native MoE expert-FFN path for Whallm's runtime.

Submodules:
  lib     ctypes binding of libwhallm_moe.so (the CUDA kernels, C ABI in include/whallm_moe.h)
  moe     PyTorch front end: Engine and the reference-shaped MoE callables
  layout  expert blob layouts and [E, ...] weight views
  waves   host-side pair scheduling (expert_waves) and the device plan's order
  synth   seeded synthetic layers of the benchmark configurations
  ep      expert parallelism over torch.distributed (NCCL)
  build   compiles the library for sm_100a
"""
__version__ = "0.1.0"
