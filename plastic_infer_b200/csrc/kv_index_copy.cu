// Slot-mapping KV write (index-copy) for the B200 paged pool.
//
// Reference behaviour: _write_kv_layer (src/plastic_infer/exec/runner_paged.py:123-129)
// and KVRequestCache.append_token (src/plastic_infer/kv/kv_store.py:140-143) store one
// token's [kv_heads, head_dim] K and V at pool[page, :, :, offset]. Here the caller
// resolves (page, offset) into a flat slot = page * page_size + offset on the host
// (BlockTable.get_page, src/plastic_infer/kv/paged.py:54-59) and the whole step's
// tokens are written by one launch.
//
// Design: one warp per token. A token's K (and V) is kv_heads rows of head_dim
// contiguous elements in the source and kv_heads rows of head_dim elements strided
// by page_size*head_dim in the pool ([P, H, S, D]). Lanes walk 16-byte vectors over
// the 2*kv_heads rows, so every warp-wide load reads 512 contiguous bytes and every
// store writes whole 256-byte row segments (full 32-byte sectors, no read-modify-write).
// Sources are streamed with L1::no_allocate; pool stores take the default policy so
// the freshly written rows stay in L2 for the attention launch that follows.
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

template <int VEC, bool kFixedLanes>
__global__ void __launch_bounds__(256) kv_index_copy_kernel(
    char* __restrict__ k_pool, char* __restrict__ v_pool, const char* __restrict__ k_new,
    const char* __restrict__ v_new, const int64_t* __restrict__ slot_mapping, int64_t n_tokens,
    int kv_heads, int row_bytes, int page_size, int64_t num_slots, int64_t src_token_stride_bytes,
    int* err) {
  using V = typename VecT<VEC>::type;
  constexpr int kPerLane = VEC == 16 ? 8 : 16;
  // Programmatic launch: nothing is read before the previous kernel has completed
  // (the new rows are its output); the next kernel may launch from here on.
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int vec_per_row = row_bytes / VEC;
  const int vec_per_tensor = kv_heads * vec_per_row;
  const int64_t head_stride = static_cast<int64_t>(page_size) * row_bytes;  // pool bytes per head
  const int64_t page_stride = head_stride * kv_heads;

  const int total = 2 * vec_per_tensor;  // vectors of one token (K then V)
  const int rows_per_pass = kFixedLanes ? 32 / vec_per_row : 0;
  const int r0 = kFixedLanes ? lane / vec_per_row : 0;
  const int64_t w0 = kFixedLanes ? static_cast<int64_t>(lane % vec_per_row) * VEC : 0;
  int64_t t = warp;
  int64_t slot = t < n_tokens ? __ldg(slot_mapping + t) : -1;
  for (; t < n_tokens; t += nwarps) {
    // Prefetch the next token's slot so its load overlaps this token's copy.
    const int64_t tn = t + nwarps;
    const int64_t next_slot = tn < n_tokens ? __ldg(slot_mapping + tn) : -1;
    const int64_t s = slot;
    slot = next_slot;
    // The source rows do not depend on the slot, so their loads go out before the slot
    // is examined and its round trip overlaps them (rows of a padding token exist too;
    // their loads are simply not stored). Only the store address waits for the slot.
    const bool store = s >= 0 && s < num_slots;
    const char* ks = k_new + t * src_token_stride_bytes;
    const char* vs = v_new + t * src_token_stride_bytes;
    // destination of this token's row group (valid only when `store`)
    auto dst_base = [&]() {
      const int64_t page = s / page_size;
      return page * page_stride + (s - page * page_size) * row_bytes;
    };

    if constexpr (kFixedLanes) {
      // 32 % vec_per_row == 0: lane `lane` always copies vector w of rows r0, r0 +
      // rows_per_pass, ... over the token's 2*kv_heads rows (K rows, then V rows), so
      // the per-vector address math has no division. All loads go out before any store.
      constexpr int kMaxRows = kPerLane;  // rows per lane handled per pass
      for (int rbase = 0; rbase < 2 * kv_heads; rbase += rows_per_pass * kMaxRows) {
        V vals[kMaxRows];
#pragma unroll
        for (int j = 0; j < kMaxRows; ++j) {
          const int r = rbase + r0 + j * rows_per_pass;
          if (r < 2 * kv_heads) {
            const bool is_v = r >= kv_heads;
            const int h = is_v ? r - kv_heads : r;
            vals[j] = load_stream<VEC>((is_v ? vs : ks) + static_cast<int64_t>(h) * row_bytes + w0);
          }
        }
        if (!store) break;
        const int64_t db = dst_base();
#pragma unroll
        for (int j = 0; j < kMaxRows; ++j) {
          const int r = rbase + r0 + j * rows_per_pass;
          if (r < 2 * kv_heads) {
            const bool is_v = r >= kv_heads;
            const int h = is_v ? r - kv_heads : r;
            *reinterpret_cast<V*>((is_v ? v_pool : k_pool) + db + h * head_stride + w0) = vals[j];
          }
        }
      }
    } else {
      // General shapes: all loads of a batch of kPerLane vectors per lane are issued
      // before any store, so a warp keeps up to 32 * kPerLane * VEC bytes in flight.
      for (int base = 0; base < total; base += 32 * kPerLane) {
        V vals[kPerLane];
#pragma unroll
        for (int j = 0; j < kPerLane; ++j) {
          const int c = base + j * 32 + lane;
          if (c < total) {
            const bool is_v = c >= vec_per_tensor;
            const int cc = is_v ? c - vec_per_tensor : c;
            const int h = cc / vec_per_row;
            const int w = cc - h * vec_per_row;
            vals[j] = load_stream<VEC>((is_v ? vs : ks) + static_cast<int64_t>(h) * row_bytes +
                                       static_cast<int64_t>(w) * VEC);
          }
        }
        if (!store) break;
        const int64_t db = dst_base();
#pragma unroll
        for (int j = 0; j < kPerLane; ++j) {
          const int c = base + j * 32 + lane;
          if (c < total) {
            const bool is_v = c >= vec_per_tensor;
            const int cc = is_v ? c - vec_per_tensor : c;
            const int h = cc / vec_per_row;
            const int w = cc - h * vec_per_row;
            *reinterpret_cast<V*>((is_v ? v_pool : k_pool) + db + h * head_stride +
                                  static_cast<int64_t>(w) * VEC) = vals[j];
          }
        }
      }
    }
    // a negative slot is padding; one past the pool is an error (the write is skipped)
    if (s >= num_slots && lane == 0) record_error(err, PI_ERR_SLOT_RANGE);
  }
}

template <int VEC>
int launch_index_copy(void* k_pool, void* v_pool, const void* k_new, const void* v_new,
                      const int64_t* slot_mapping, int64_t n_tokens, int kv_heads, int row_bytes,
                      int page_size, int64_t num_slots, int64_t src_stride_bytes, int* err,
                      cudaStream_t stream) {
  constexpr int kThreads = 256;
  constexpr int kWarpsPerBlock = kThreads / 32;
  const int sms = device_sm_count();
  int64_t blocks = (n_tokens + kWarpsPerBlock - 1) / kWarpsPerBlock;
  const int64_t cap = static_cast<int64_t>(sms) * 16;  // grid-stride beyond 16 CTAs per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const bool fixed = (32 % (row_bytes / VEC)) == 0;
  const dim3 grid(static_cast<unsigned>(blocks));
  const cudaError_t e = launch_kernel(
      fixed ? kv_index_copy_kernel<VEC, true> : kv_index_copy_kernel<VEC, false>, grid,
      dim3(kThreads), 0, stream, static_cast<char*>(k_pool), static_cast<char*>(v_pool),
      static_cast<const char*>(k_new), static_cast<const char*>(v_new), slot_mapping, n_tokens,
      kv_heads, row_bytes, page_size, num_slots, src_stride_bytes, err);
  return cuda_status(e);
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
  if (fits(16))
    return launch_index_copy<16>(k_pool, v_pool, k_new, v_new, slot_mapping, n_tokens, kv_heads,
                                 row_bytes, page_size, num_slots, stride_bytes, err, stream);
  if (fits(8))
    return launch_index_copy<8>(k_pool, v_pool, k_new, v_new, slot_mapping, n_tokens, kv_heads,
                                row_bytes, page_size, num_slots, stride_bytes, err, stream);
  if (fits(4))
    return launch_index_copy<4>(k_pool, v_pool, k_new, v_new, slot_mapping, n_tokens, kv_heads,
                                row_bytes, page_size, num_slots, stride_bytes, err, stream);
  if (fits(2))
    return launch_index_copy<2>(k_pool, v_pool, k_new, v_new, slot_mapping, n_tokens, kv_heads,
                                row_bytes, page_size, num_slots, stride_bytes, err, stream);
  return PI_ERR_MISALIGNED;
}
