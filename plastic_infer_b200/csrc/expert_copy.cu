// MoE expert-slot copy: for every bank b and i < n,
//   dst_b[dst_indices[i]] = src_b[src_indices[i]]        (rows of feat_bytes[b] bytes)
// in one launch. The banks' base addresses and row sizes are small device arrays, so the
// launch is CUDA-graph safe; n is read from the device (`num_indices`) when given.
//
// Replaces the fused multi-bank copy of the reference's MoE slot cache
// (fast_index_copy_multi_jit, src/plastic_infer/kernel/fast_index_copy.py:190-244; kernel
// src/plastic_infer/kernel/csrc/jit/fast_index_copy.cuh:436-503), called by
// OffloadMoeCache.copy_missing (src/plastic_infer/moe/offload_cache.py:998-1012). The source
// banks are pinned host memory read through their device alias, so the copy is bound by
// the host link.
//
// The reference launches 8 blocks of 1024 threads per bank whatever n is, each thread
// moving one 16-byte unit per iteration (one load, then its store). Here every (bank,
// row) is cut into 4 KiB chunks spread over all warps of a full-GPU grid; a lane issues
// its 8 loads of a chunk before any store, so a warp keeps 4 KiB of host reads in flight.
#include "pi_common.cuh"

namespace pi {
namespace {

constexpr int kChunk = 4096;       // bytes of one work item
constexpr int kMaxBanks = 32;

struct ExpertCopyParams {
  const int64_t* dst_ptrs;    // [num_banks] device: slot-cache base addresses
  const int64_t* src_ptrs;    // [num_banks] device: host-bank device aliases
  const int64_t* feat_bytes;  // [num_banks] device: bytes per row (multiple of 16)
  const void* dst_indices;    // [length]
  const void* src_indices;    // [length]
  const int64_t* valid_length;  // [1] or null
  int64_t length;
  int num_banks;
  int* err;
};

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <typename Id>
__global__ void __launch_bounds__(256) expert_slot_copy_kernel(const __grid_constant__ ExpertCopyParams p) {
  pdl_wait();  // the indices and the valid length are the previous kernel's output
  pdl_trigger();
  __shared__ int64_t s_feat[kMaxBanks];
  __shared__ int64_t s_off[kMaxBanks + 1];  // first work item of each bank
  __shared__ int64_t s_chunks[kMaxBanks];
  int64_t n = p.valid_length != nullptr ? __ldg(p.valid_length) : p.length;
  if (n > p.length) n = p.length;
  if (n <= 0) return;
  if (threadIdx.x == 0) {
    int64_t off = 0;
    for (int b = 0; b < p.num_banks; ++b) {
      int64_t feat = __ldg(p.feat_bytes + b);
      const bool ok = feat > 0 && feat % 16 == 0 && __ldg(p.dst_ptrs + b) % 16 == 0 &&
                      __ldg(p.src_ptrs + b) % 16 == 0;
      if (!ok) {
        if (blockIdx.x == 0) record_error(p.err, PI_ERR_MISALIGNED);
        feat = 0;  // bank skipped
      }
      s_feat[b] = feat;
      s_chunks[b] = (feat + kChunk - 1) / kChunk;
      s_off[b] = off;
      off += n * s_chunks[b];
    }
    s_off[p.num_banks] = off;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t total = s_off[p.num_banks];
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const Id* di = static_cast<const Id*>(p.dst_indices);
  const Id* si = static_cast<const Id*>(p.src_indices);
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < total;
       w += nwarps) {
    int b = 0;
    while (b + 1 < p.num_banks && s_off[b + 1] <= w) ++b;
    const int64_t chunks = s_chunks[b];
    const int64_t rel = w - s_off[b];
    const int64_t row = rel / chunks;
    const int64_t c = rel - row * chunks;
    const int64_t pd = static_cast<int64_t>(__ldg(di + row));
    const int64_t ps = static_cast<int64_t>(__ldg(si + row));
    if (pd < 0 || ps < 0) {
      if (lane == 0) record_error(p.err, PI_ERR_SLOT_RANGE);
      continue;
    }
    const int64_t feat = s_feat[b];
    const int64_t begin = c * kChunk;
    const int64_t bytes = feat - begin < kChunk ? feat - begin : kChunk;
    const char* src = reinterpret_cast<const char*>(__ldg(p.src_ptrs + b)) + ps * feat + begin;
    char* dst = reinterpret_cast<char*>(__ldg(p.dst_ptrs + b)) + pd * feat + begin;
    uint4 v[kChunk / 512];
#pragma unroll
    for (int k = 0; k < kChunk / 512; ++k) {
      const int64_t o = static_cast<int64_t>(k) * 512 + lane * 16;
      if (o < bytes) v[k] = ld_stream16(src + o);
    }
#pragma unroll
    for (int k = 0; k < kChunk / 512; ++k) {
      const int64_t o = static_cast<int64_t>(k) * 512 + lane * 16;
      if (o < bytes) *reinterpret_cast<uint4*>(dst + o) = v[k];
    }
  }
}

}  // namespace
}  // namespace pi

extern "C" int pi_expert_slot_copy(const int64_t* dst_ptrs, const int64_t* src_ptrs,
                                   const int64_t* feat_bytes, int num_banks,
                                   const void* dst_indices, const void* src_indices,
                                   int64_t length, const int64_t* num_indices, int use_int32,
                                   int* err, cudaStream_t stream) {
  using namespace pi;
  if (num_banks < 0 || num_banks > kMaxBanks || length < 0) return PI_ERR_BAD_SHAPE;
  if (num_banks == 0 || length == 0) return PI_OK;
  if (!dst_ptrs || !src_ptrs || !feat_bytes || !dst_indices || !src_indices)
    return PI_ERR_NULL_POINTER;
  if (!aligned(dst_ptrs, 8) || !aligned(src_ptrs, 8) || !aligned(feat_bytes, 8) ||
      (num_indices != nullptr && !aligned(num_indices, 8)) ||
      !aligned(dst_indices, use_int32 ? 4 : 8) || !aligned(src_indices, use_int32 ? 4 : 8))
    return PI_ERR_MISALIGNED;
  ExpertCopyParams p;
  p.dst_ptrs = dst_ptrs;
  p.src_ptrs = src_ptrs;
  p.feat_bytes = feat_bytes;
  p.dst_indices = dst_indices;
  p.src_indices = src_indices;
  p.valid_length = num_indices;
  p.length = length;
  p.num_banks = num_banks;
  p.err = err;
  // One full-GPU wave: 4 CTAs of 8 warps per SM, each warp 4 KiB of loads in flight.
  const dim3 grid(static_cast<unsigned>(device_sm_count() * 4));
  return cuda_status(use_int32 ? launch_kernel(expert_slot_copy_kernel<int32_t>, grid, dim3(256), 0,
                                               stream, p)
                               : launch_kernel(expert_slot_copy_kernel<int64_t>, grid, dim3(256), 0,
                                               stream, p));
}
