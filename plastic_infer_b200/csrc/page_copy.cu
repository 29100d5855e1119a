// Page moves between the paged pool and contiguous staging buffers, and the
// contiguous per-request gather used by gather_paged_kv.
//
// Reference behaviour:
//   - KVStore.sink_completed_chunks copies each (layer, page) of a completed chunk
//     with k_pages[phys].to("cpu") into k_chunk[layer, :, :, t0:t1]
//     (src/plastic_infer/kv/kv_store.py:258-269);
//   - KVStore.load_prefix copies them back with .to(device) into freshly
//     allocated pages (src/plastic_infer/kv/kv_store.py:311-321);
//   - gather_paged_kv index_selects the block table's pages and permutes them to
//     [tokens, heads, head_dim] (src/plastic_infer/exec/attention.py:133-148).
// Here one launch moves a whole list of pages between the pool and a staging buffer
// laid out exactly like the host chunk, so the host<->device leg is one large
// cudaMemcpyAsync issued by the caller on a side stream.
//
// All three are pure byte moves bound by HBM: 16-byte vector loads/stores, one
// warp per (page, head) tile, grid sized to a multiple of the SM count.
#include "pi_common.cuh"

namespace pi {
namespace {

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Copy `bytes` (a multiple of 16) from src to dst with one warp, 4 vectors in flight
// per lane.
__device__ __forceinline__ void warp_copy16(char* __restrict__ dst, const char* __restrict__ src,
                                            int64_t bytes, int lane) {
  const int64_t nvec = bytes >> 4;
  int64_t i = lane;
  for (; i + 96 < nvec; i += 128) {
    const uint4 a = ld_stream16(src + (i << 4));
    const uint4 b = ld_stream16(src + ((i + 32) << 4));
    const uint4 c = ld_stream16(src + ((i + 64) << 4));
    const uint4 d = ld_stream16(src + ((i + 96) << 4));
    *reinterpret_cast<uint4*>(dst + (i << 4)) = a;
    *reinterpret_cast<uint4*>(dst + ((i + 32) << 4)) = b;
    *reinterpret_cast<uint4*>(dst + ((i + 64) << 4)) = c;
    *reinterpret_cast<uint4*>(dst + ((i + 96) << 4)) = d;
  }
  for (; i < nvec; i += 32) {
    *reinterpret_cast<uint4*>(dst + (i << 4)) = ld_stream16(src + (i << 4));
  }
}

// to_pool == false: staging <- pool (gather); true: pool <- staging (scatter).
template <bool kToPool>
__global__ void __launch_bounds__(256) page_move_kernel(char* __restrict__ pool_or_dst,
                                                        const char* __restrict__ src,
                                                        const int32_t* __restrict__ page_ids,
                                                        int64_t n_pages, int kv_heads,
                                                        int64_t tile_bytes, int ppg,
                                                        int64_t num_pages, int* err) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t n_tiles = n_pages * kv_heads;
  for (int64_t tile = warp; tile < n_tiles; tile += nwarps) {
    const int64_t i = tile / kv_heads;
    const int h = static_cast<int>(tile - i * kv_heads);
    const int64_t pid = __ldg(page_ids + i);
    if (pid < 0 || pid >= num_pages) {
      if (lane == 0) record_error(err, PI_ERR_PAGE_RANGE);
      continue;
    }
    const int64_t g = i / ppg;
    const int64_t j = i - g * ppg;
    const int64_t stage_off = ((g * kv_heads + h) * ppg + j) * tile_bytes;
    const int64_t pool_off = (pid * kv_heads + h) * tile_bytes;
    if (kToPool) {
      warp_copy16(pool_or_dst + pool_off, src + stage_off, tile_bytes, lane);
    } else {
      warp_copy16(pool_or_dst + stage_off, src + pool_off, tile_bytes, lane);
    }
  }
}

// out[t, h, :] = pool[bt[t / S], h, t % S, :]; one warp per token, vector width VEC.
template <typename V>
__global__ void __launch_bounds__(256) paged_kv_gather_kernel(
    char* __restrict__ out, const char* __restrict__ pool, const int32_t* __restrict__ block_table,
    int64_t num_tokens, int kv_heads, int row_bytes, int page_size, int64_t num_pages, int* err) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  constexpr int VB = sizeof(V);
  const int vec_per_row = row_bytes / VB;
  const int nvec = kv_heads * vec_per_row;
  for (int64_t t = warp; t < num_tokens; t += nwarps) {
    const int64_t pid = __ldg(block_table + t / page_size);
    const int64_t off = t % page_size;
    char* dst = out + t * static_cast<int64_t>(kv_heads) * row_bytes;
    if (pid < 0 || pid >= num_pages) {
      if (lane == 0) record_error(err, PI_ERR_PAGE_RANGE);
      for (int c = lane; c < nvec; c += 32) reinterpret_cast<V*>(dst)[c] = V{};
      continue;
    }
    const char* base = pool + (pid * kv_heads) * static_cast<int64_t>(page_size) * row_bytes +
                       off * row_bytes;
    for (int c = lane; c < nvec; c += 32) {
      const int h = c / vec_per_row;
      const int w = c - h * vec_per_row;
      const V v = *reinterpret_cast<const V*>(
          base + static_cast<int64_t>(h) * page_size * row_bytes + static_cast<int64_t>(w) * VB);
      reinterpret_cast<V*>(dst)[c] = v;
    }
  }
}

unsigned grid_for(int64_t warps_needed) {
  const int64_t per_block = 8;
  int64_t blocks = (warps_needed + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<unsigned>(blocks);
}

template <bool kToPool>
int page_move(void* dst, const void* src, const int32_t* page_ids, int64_t n_pages, int kv_heads,
              int64_t tile_bytes, int ppg, int64_t num_pages, int* err, cudaStream_t stream) {
  if (n_pages < 0 || kv_heads <= 0 || tile_bytes <= 0 || ppg <= 0 || num_pages < 0)
    return PI_ERR_BAD_SHAPE;
  if (n_pages == 0) return PI_OK;
  if (!dst || !src || !page_ids) return PI_ERR_NULL_POINTER;
  if (tile_bytes % 16 != 0 || !aligned(dst, 16) || !aligned(src, 16) || !aligned(page_ids, 4))
    return PI_ERR_MISALIGNED;
  page_move_kernel<kToPool><<<grid_for(n_pages * kv_heads), 256, 0, stream>>>(
      static_cast<char*>(dst), static_cast<const char*>(src), page_ids, n_pages, kv_heads,
      tile_bytes, ppg, num_pages, err);
  return cuda_status(cudaGetLastError());
}

}  // namespace
}  // namespace pi

extern "C" int pi_page_gather(void* staging, const void* pool, const int32_t* page_ids,
                              int64_t n_pages, int kv_heads, int64_t tile_bytes,
                              int pages_per_group, int64_t num_pages, int* err,
                              cudaStream_t stream) {
  return pi::page_move<false>(staging, pool, page_ids, n_pages, kv_heads, tile_bytes,
                              pages_per_group, num_pages, err, stream);
}

extern "C" int pi_page_scatter(void* pool, const void* staging, const int32_t* page_ids,
                               int64_t n_pages, int kv_heads, int64_t tile_bytes,
                               int pages_per_group, int64_t num_pages, int* err,
                               cudaStream_t stream) {
  return pi::page_move<true>(pool, staging, page_ids, n_pages, kv_heads, tile_bytes,
                             pages_per_group, num_pages, err, stream);
}

extern "C" int pi_paged_kv_gather(void* out, const void* pool, const int32_t* block_table,
                                  int64_t num_tokens, int kv_heads, int head_dim, int page_size,
                                  int64_t num_pages, int dtype, int* err, cudaStream_t stream) {
  using namespace pi;
  const int eb = elem_bytes_of(dtype);
  if (eb == 0) return PI_ERR_UNSUPPORTED;
  if (num_tokens < 0 || kv_heads <= 0 || head_dim <= 0 || page_size <= 0 || num_pages < 0)
    return PI_ERR_BAD_SHAPE;
  if (num_tokens == 0) return PI_OK;
  if (!out || !pool || !block_table) return PI_ERR_NULL_POINTER;
  const int row_bytes = head_dim * eb;
  const unsigned grid = grid_for(num_tokens);
  const bool a16 = row_bytes % 16 == 0 && aligned(out, 16) && aligned(pool, 16);
  const bool a4 = row_bytes % 4 == 0 && aligned(out, 4) && aligned(pool, 4);
  if (a16) {
    paged_kv_gather_kernel<uint4><<<grid, 256, 0, stream>>>(
        static_cast<char*>(out), static_cast<const char*>(pool), block_table, num_tokens, kv_heads,
        row_bytes, page_size, num_pages, err);
  } else if (a4) {
    paged_kv_gather_kernel<uint32_t><<<grid, 256, 0, stream>>>(
        static_cast<char*>(out), static_cast<const char*>(pool), block_table, num_tokens, kv_heads,
        row_bytes, page_size, num_pages, err);
  } else {
    paged_kv_gather_kernel<uint16_t><<<grid, 256, 0, stream>>>(
        static_cast<char*>(out), static_cast<const char*>(pool), block_table, num_tokens, kv_heads,
        row_bytes, page_size, num_pages, err);
  }
  return cuda_status(cudaGetLastError());
}
