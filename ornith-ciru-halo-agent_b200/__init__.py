"""B200-native routed mixture-of-experts layer of Ornith (drop-in for the
routed path of ciru-ai/ornith-ciru-halo-agent).

Modules:
  native     ctypes binding of libornith_moe_b200.so and the torch custom ops
  runtime    workspace arena and per-layer sticky error flags
  lifecycle  per-step flag snapshots and worker poisoning (failure detection)
  method     packed-weight methods and strict checkpoint loaders
  ep         expert parallelism over torch.distributed
  synthetic  seeded inputs with the benchmark configurations' shapes
  build      nvcc build of the in-tree CUDA library

The package directory name contains hyphens; it is imported under the name
`ornith_b200` by __graft_entry__.load_package().
"""
ABI_VERSION = 1
