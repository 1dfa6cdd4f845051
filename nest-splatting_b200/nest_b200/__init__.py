"""B200-native (sm_100a) implementation of nest-splatting's render hot path.

Modules:
  _lib    ctypes bindings of libnest_b200.so (the C-ABI in include/nest_b200.h)
  raster  torch-facing wrappers: rasterizer forward, MLP, RVQ decode, radix sort
  frame   the fused RVQ-driven frame (decode -> rasterize -> MLP)
  camera  pinhole cameras in the reference's conventions
  synth   seeded synthetic scenes of the benchmark configurations
  views   multi-view batches sharded by camera over torch.distributed ranks
"""
__all__ = ["_lib", "raster", "frame", "camera", "synth"]
