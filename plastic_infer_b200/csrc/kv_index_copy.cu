// Slot-mapping KV write (index-copy) for the B200 paged pool.
//
// Reference behaviour: _write_kv_layer (src/plastic_infer/exec/runner_paged.py:123-129)
// and KVRequestCache.append_token (src/plastic_infer/kv/kv_store.py:140-143) store one
// token's [kv_heads, head_dim] K and V at pool[page, :, :, offset]. Here the caller
// resolves (page, offset) into a flat slot = page * page_size + offset on the host
// (BlockTable.get_page, src/plastic_infer/kv/paged.py:54-59) and the whole step's
// tokens are written by one launch.
//
// Design: the unit of work is one warp-wide chunk of one token's bytes. A token's K
// and V are 2*kv_heads rows of head_dim contiguous elements in the source and
// 2*kv_heads rows strided by page_size*head_dim in the pool ([P, H, S, D]); seen as
// VEC-byte vectors (K rows, then V rows) they are cut into chunks of 32 vectors, lane l
// copying vector l of its chunk. At the 8B shape (8 heads x 256-byte rows, bf16) a token
// is 8 chunks of 512 bytes, so even a 64-token step is 512 warps over 128 CTAs instead
// of 64 warps on 8 SMs: the step's DRAM round trips run on most of the GPU at once.
// Every warp-wide load reads 512 contiguous bytes and every store writes whole 256-byte
// row segments (full 32-byte sectors, no read-modify-write).
//
// A warp takes UNROLL consecutive chunks per pass (one token's when the token has a
// multiple of UNROLL chunks: one slot load) and issues their slot and source loads before
// any store, so one pass costs one DRAM round trip. The host uses one chunk per warp for
// the smallest launches and two otherwise, with a grid-stride loop beyond one resident
// wave, so successive passes of a warp overlap the loads of one with the stores of the
// last (see launch_index_copy for the measurements). Sources are streamed with L1::no_allocate; pool stores
// take the default policy so the freshly written rows stay in L2 for the attention
// launch that follows.
#include "pi_common.cuh"

namespace pi {
namespace {

template <int VEC>
struct VecT;
template <>
struct VecT<16> {
  using type = uint4;
};
template <>
struct VecT<8> {
  using type = uint2;
};
template <>
struct VecT<4> {
  using type = uint32_t;
};
template <>
struct VecT<2> {
  using type = uint16_t;
};

template <int VEC>
__device__ __forceinline__ typename VecT<VEC>::type load_stream(const void* p) {
  using V = typename VecT<VEC>::type;
  if constexpr (VEC == 16) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
  } else {
    return __ldg(reinterpret_cast<const V*>(p));
  }
}

struct CopyArgs {
  char* k_pool;
  char* v_pool;
  const char* k_new;
  const char* v_new;
  const int64_t* slot_mapping;
  int* err;
  int64_t n_chunks;       // n_tokens * chunks_per_token
  int64_t num_slots;
  int64_t src_stride;     // bytes between consecutive tokens of the source
  int64_t head_stride;    // pool bytes between heads of one page (page_size * row_bytes)
  int64_t page_stride;    // pool bytes per page (kv_heads * head_stride)
  int chunks_per_token;   // ceil(2 * kv_heads * vec_per_row / 32)
  int vec_per_tensor;     // kv_heads * vec_per_row (vectors of one token's K)
  int vec_per_row;
  int kv_heads;
  int row_shift;          // log2(vec_per_row) when it is a power of two, else -1
  int row_bytes;
  int page_size;
};

constexpr int kCopyThreads = 128;

// One VEC-byte vector of a token's rows: vector v (0 .. 2 * vec_per_tensor) is vector w
// of row r, rows 0..H-1 being K heads and H..2H-1 V heads.
struct RowVec {
  int head;
  int w;
  bool is_v;
};

__device__ __forceinline__ RowVec row_vec(const CopyArgs& a, int v) {
  const int r = a.row_shift >= 0 ? v >> a.row_shift : v / a.vec_per_row;
  const bool is_v = r >= a.kv_heads;
  return RowVec{is_v ? r - a.kv_heads : r, v - r * a.vec_per_row, is_v};
}

// A token's K (and V) rows are contiguous in the source, so vector v of the K rows sits
// at byte v * VEC of the token's K, and vector v >= vec_per_tensor at byte
// (v - vec_per_tensor) * VEC of its V.
template <int VEC>
__device__ __forceinline__ typename VecT<VEC>::type load_vec(const CopyArgs& a, int64_t t, int v) {
  const bool is_v = v >= a.vec_per_tensor;
  return load_stream<VEC>((is_v ? a.v_new : a.k_new) + t * a.src_stride +
                          static_cast<int64_t>(is_v ? v - a.vec_per_tensor : v) * VEC);
}

template <int VEC>
__device__ __forceinline__ void store_vec(const CopyArgs& a, int64_t s, bool small, int v,
                                          typename VecT<VEC>::type val) {
  using V = typename VecT<VEC>::type;
  const RowVec rv = row_vec(a, v);
  int64_t page, pos;
  if (small) {
    const unsigned us = static_cast<unsigned>(s);
    const unsigned pg = us / static_cast<unsigned>(a.page_size);
    page = pg;
    pos = us - pg * static_cast<unsigned>(a.page_size);
  } else {
    page = s / a.page_size;
    pos = s - page * a.page_size;
  }
  char* dst = (rv.is_v ? a.v_pool : a.k_pool) + page * a.page_stride + rv.head * a.head_stride +
              pos * a.row_bytes + static_cast<int64_t>(rv.w) * VEC;
  *reinterpret_cast<V*>(dst) = val;
}

// kWhole: chunks_per_token is a multiple of UNROLL, so a unit is UNROLL chunks of one
// token and needs one slot; otherwise a unit may span tokens and loads a slot per chunk.
template <int VEC, int UNROLL, bool kWhole>
__global__ void __launch_bounds__(kCopyThreads) kv_index_copy_kernel(const CopyArgs a) {
  using V = typename VecT<VEC>::type;
  // Programmatic launch: nothing is read before the previous kernel has completed
  // (the new rows are its output); the next kernel may launch from here on.
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  // 32-bit index arithmetic whenever the sizes allow it (always, for real pools)
  const bool small = a.num_slots <= 0x7fffffff && a.n_chunks <= 0x7fffffff;
  const int64_t n_units = (a.n_chunks + UNROLL - 1) / UNROLL;
  const int nvec = 2 * a.vec_per_tensor;

  for (int64_t u = warp; u < n_units; u += nwarps) {
    // chunks u * UNROLL ... u * UNROLL + UNROLL - 1 of the token-major chunk sequence
    const int64_t first = u * UNROLL;
    int64_t t;
    int c;
    if (small) {
      const unsigned f = static_cast<unsigned>(first);
      const unsigned tt = f / static_cast<unsigned>(a.chunks_per_token);
      t = tt;
      c = static_cast<int>(f - tt * static_cast<unsigned>(a.chunks_per_token));
    } else {
      t = first / a.chunks_per_token;
      c = static_cast<int>(first - t * a.chunks_per_token);
    }
    V vals[UNROLL];
    // All slot and source loads of the unit go out before any store. The source rows
    // do not depend on the slot, so the two round trips overlap.
    if constexpr (kWhole) {
      const int64_t s = __ldg(a.slot_mapping + t);  // one address per warp: a broadcast
#pragma unroll
      for (int j = 0; j < UNROLL; ++j) {
        const int v = (c + j) * 32 + lane;
        if (v < nvec) vals[j] = load_vec<VEC>(a, t, v);
      }
      if (c == 0 && lane == 0 && s >= a.num_slots) record_error(a.err, PI_ERR_SLOT_RANGE);
      if (s < 0 || s >= a.num_slots) continue;  // padding, or out of range (skipped)
#pragma unroll
      for (int j = 0; j < UNROLL; ++j) {
        const int v = (c + j) * 32 + lane;
        if (v < nvec) store_vec<VEC>(a, s, small, v, vals[j]);
      }
    } else {
      int64_t slot[UNROLL];
      int chunk[UNROLL];
#pragma unroll
      for (int j = 0; j < UNROLL; ++j) {
        slot[j] = -1;
        chunk[j] = c;
        if (first + j < a.n_chunks) {
          slot[j] = __ldg(a.slot_mapping + t);
          const int v = c * 32 + lane;
          if (v < nvec) vals[j] = load_vec<VEC>(a, t, v);
          // a negative slot is padding; one past the pool is an error (the write is skipped)
          if (c == 0 && lane == 0 && slot[j] >= a.num_slots)
            record_error(a.err, PI_ERR_SLOT_RANGE);
        }
        if (++c == a.chunks_per_token) {
          c = 0;
          ++t;
        }
      }
#pragma unroll
      for (int j = 0; j < UNROLL; ++j) {
        const int v = chunk[j] * 32 + lane;
        if (slot[j] >= 0 && slot[j] < a.num_slots && v < nvec)
          store_vec<VEC>(a, slot[j], small, v, vals[j]);
      }
    }
  }
}

template <int VEC, int UNROLL, bool kWhole>
int launch_unrolled(const CopyArgs& a, int64_t warps, int ctas_per_sm, cudaStream_t stream) {
  int64_t blocks = (warps + kCopyThreads / 32 - 1) / (kCopyThreads / 32);
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * ctas_per_sm;
  if (blocks > cap) blocks = cap;  // grid-stride beyond one resident wave
  if (blocks < 1) blocks = 1;
  return cuda_status(launch_kernel(kv_index_copy_kernel<VEC, UNROLL, kWhole>,
                                   dim3(static_cast<unsigned>(blocks)), dim3(kCopyThreads), 0,
                                   stream, a));
}

// Resident CTAs per SM of one instance on the current device (cached per device).
template <int VEC, int UNROLL, bool kWhole>
int resident_ctas() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 8;
  if (cache[dev] == 0) {
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kv_index_copy_kernel<VEC, UNROLL, kWhole>,
                                                      kCopyThreads, 0) != cudaSuccess ||
        occ < 1) {
      (void)cudaGetLastError();
      occ = 8;
    }
    cache[dev] = occ;
  }
  return cache[dev];
}

template <int VEC, int UNROLL>
int launch_with(const CopyArgs& a, cudaStream_t stream) {
  const int64_t units = (a.n_chunks + UNROLL - 1) / UNROLL;
  if (a.chunks_per_token % UNROLL == 0)
    return launch_unrolled<VEC, UNROLL, true>(a, units, resident_ctas<VEC, UNROLL, true>(), stream);
  return launch_unrolled<VEC, UNROLL, false>(a, units, resident_ctas<VEC, UNROLL, false>(), stream);
}

template <int VEC>
int launch_index_copy(CopyArgs a, cudaStream_t stream) {
  // One chunk per warp for the smallest launches (up to 1,024 chunks: a 128-token step of
  // the 8B shape), which then spread over the most SMs; two consecutive chunks per warp
  // and pass otherwise, with a grid-stride loop beyond one resident wave. Measured on B200
  // (CUDA graphs of back-to-back plain launches, L2 flushed): at 512 / 4,096 / 65,536
  // tokens two chunks per pass took 2.43 / 7.72 / 93.6 us against 2.80 / 7.75-8.59 /
  // 95.8-104.5 us for one, four or eight; at 64 tokens one chunk took 1.73 us against 1.87
  // for two. With programmatic launch between the launches the 512-token case is within
  // 3 % either way (2.95 against 2.87 us).
  if (a.n_chunks <= 1024) return launch_with<VEC, 1>(a, stream);
  return launch_with<VEC, 2>(a, stream);
}

}  // namespace
}  // namespace pi

extern "C" int pi_kv_index_copy(void* k_pool, void* v_pool, const void* k_new, const void* v_new,
                                const int64_t* slot_mapping, int64_t n_tokens, int kv_heads,
                                int head_dim, int page_size, int64_t num_slots, int dtype,
                                int64_t src_token_stride, int* err, cudaStream_t stream) {
  using namespace pi;
  const int eb = elem_bytes_of(dtype);
  if (eb == 0) return PI_ERR_UNSUPPORTED;
  if (n_tokens < 0 || kv_heads <= 0 || head_dim <= 0 || page_size <= 0 || num_slots < 0)
    return PI_ERR_BAD_SHAPE;
  if (src_token_stride < static_cast<int64_t>(kv_heads) * head_dim) return PI_ERR_BAD_SHAPE;
  if (n_tokens == 0) return PI_OK;
  if (!k_pool || !v_pool || !k_new || !v_new || !slot_mapping) return PI_ERR_NULL_POINTER;
  if (!aligned(slot_mapping, 8)) return PI_ERR_MISALIGNED;
  const int row_bytes = head_dim * eb;
  const int64_t stride_bytes = src_token_stride * eb;
  // Widest vector that divides every address and stride involved.
  auto fits = [&](int v) {
    return row_bytes % v == 0 && stride_bytes % v == 0 && aligned(k_pool, v) &&
           aligned(v_pool, v) && aligned(k_new, v) && aligned(v_new, v);
  };
  const int vec = fits(16) ? 16 : fits(8) ? 8 : fits(4) ? 4 : fits(2) ? 2 : 0;
  if (vec == 0) return PI_ERR_MISALIGNED;
  CopyArgs a;
  a.k_pool = static_cast<char*>(k_pool);
  a.v_pool = static_cast<char*>(v_pool);
  a.k_new = static_cast<const char*>(k_new);
  a.v_new = static_cast<const char*>(v_new);
  a.slot_mapping = slot_mapping;
  a.err = err;
  a.num_slots = num_slots;
  a.src_stride = stride_bytes;
  a.row_bytes = row_bytes;
  a.page_size = page_size;
  a.head_stride = static_cast<int64_t>(page_size) * row_bytes;
  a.page_stride = a.head_stride * kv_heads;
  a.vec_per_row = row_bytes / vec;
  a.kv_heads = kv_heads;
  a.row_shift = (a.vec_per_row & (a.vec_per_row - 1)) == 0 ? __builtin_ctz(a.vec_per_row) : -1;
  const int64_t vec_per_tensor = static_cast<int64_t>(kv_heads) * a.vec_per_row;
  if (2 * vec_per_tensor > (int64_t{1} << 30)) return PI_ERR_UNSUPPORTED;
  a.vec_per_tensor = static_cast<int>(vec_per_tensor);
  a.chunks_per_token = static_cast<int>((2 * vec_per_tensor + 31) / 32);
  if (n_tokens > (int64_t{1} << 62) / a.chunks_per_token) return PI_ERR_BAD_SHAPE;
  a.n_chunks = n_tokens * a.chunks_per_token;
  switch (vec) {
    case 16: return launch_index_copy<16>(a, stream);
    case 8: return launch_index_copy<8>(a, stream);
    case 4: return launch_index_copy<4>(a, stream);
    default: return launch_index_copy<2>(a, stream);
  }
}
