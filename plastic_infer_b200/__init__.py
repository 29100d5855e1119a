"""plastic_infer_b200: B200-native (sm_100a) paged-KV decode path for plastic-infer.

Three hand-written CUDA kernels behind a C ABI (include/plastic_kv.h,
plastic_infer_b200/csrc/) and the reference's Python API on top:

  kernels          batched entry points (index-copy, paged decode attention,
                   page gather/scatter, contiguous gather)
  kv               KVConfig / KVPagedStorage / KVRequestCache / KVStore, BlockTable,
                   PageAllocator, chunk keys (same interface as plastic_infer.kv)
  exec             gather_paged_kv / paged_attention_v1 and the paged dense runner
                   (same interface as plastic_infer.exec)
  decode           batched multi-request decode driver
  dist             KV-head sharding across GPUs with an all-gather before o_proj
  install          rebinding hook that drops this path into a plastic-infer install
"""

__version__ = "0.1.0"
