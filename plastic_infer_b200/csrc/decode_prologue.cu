// Fused decode prologue: per-head RMSNorm (QK-norm, optional) + rotary embedding of the
// step's query and key rows, and the slot-mapping write of the new K/V rows into the
// page pools, in one launch.
//
// Replaces, for one decode step of one layer, the per-op sequence of the reference
// runners: qk_norm (src/plastic_infer/exec/attention.py:83-95, Qwen3-style, before RoPE),
// rope_positions on q and k (attention.py:23-49) over a table from build_rope_cache
// (attention.py:52-74), then _write_kv_layer (src/plastic_infer/exec/runner_paged.py:112-129).
// The reference builds the cos/sin table in the model dtype (bf16 in bf16 runs) every
// step (runner_paged.py:231-232); here every angle is pos * inv_freq[j] in fp32, the
// product the reference's fp32 table holds, and cos/sin come from sincosf.
//
// One warp per (request, head) row; lane l holds elements [l*E, l*E + E), E = D / 32.
// RoPE pairs element j with j + D/2 (rotate_half), which always sits 16 lanes away.
#include "pi_common.cuh"

namespace pi {
namespace {

struct PrologueParams {
  void* q_out;                // [B, Hq, D] pool dtype, request stride q_out_stride
  char* k_pool;               // physical [P, Hkv, S, D]
  char* v_pool;
  const void* q_in;           // [B, Hq, D] input dtype, request stride q_in_stride
  const void* k_in;           // [B, Hkv, D], request stride kv_in_stride
  const void* v_in;
  const void* q_norm_w;       // [D] input dtype, or null (no QK-norm)
  const void* k_norm_w;
  const float* inv_freq;      // [D / 2]
  const int64_t* positions;   // [B]
  const int64_t* slot_mapping;  // [B], < 0: no K/V write for that request
  int64_t q_out_stride;
  int64_t q_in_stride;
  int64_t kv_in_stride;
  int64_t num_slots;
  float eps;
  int batch, hq, hkv, page_size;
  int* err;
};

// E elements per lane (D = 32 E), input type Ti, pool/output type To.
template <typename Ti, typename To, int E>
__global__ void __launch_bounds__(256) decode_prologue_kernel(const PrologueParams p) {
  pdl_wait();  // the inputs are the previous kernel's outputs (the projections)
  pdl_trigger();
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int rows_per_req = p.hq + 2 * p.hkv;  // q heads, then k heads, then v heads
  const int64_t rows = static_cast<int64_t>(p.batch) * rows_per_req;
  const int d0 = lane * E;
  const bool upper = lane >= 16;  // holds elements j + D/2 of the rotate_half pairs

  for (int64_t r = warp; r < rows; r += nwarps) {
    const int b = static_cast<int>(r / rows_per_req);
    const int h = static_cast<int>(r - static_cast<int64_t>(b) * rows_per_req);
    const bool is_q = h < p.hq;
    const bool is_v = h >= p.hq + p.hkv;
    const int kh = is_q ? h : (is_v ? h - p.hq - p.hkv : h - p.hq);
    const int64_t slot = is_q ? 0 : __ldg(p.slot_mapping + b);
    if (!is_q && slot < 0) continue;  // no new row for this request
    if (!is_q && slot >= p.num_slots) {
      if (lane == 0) record_error(p.err, PI_ERR_SLOT_RANGE);
      continue;
    }
    const Ti* src = is_q ? static_cast<const Ti*>(p.q_in) + b * p.q_in_stride + kh * D
                         : static_cast<const Ti*>(is_v ? p.v_in : p.k_in) + b * p.kv_in_stride +
                               kh * D;
    float x[E];
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = to_f32(src[d0 + e]);

    if (!is_v) {
      // QK-norm: x / sqrt(mean(x^2) + eps) * w over the head's D elements.
      const Ti* w = static_cast<const Ti*>(is_q ? p.q_norm_w : p.k_norm_w);
      if (w != nullptr) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) ss += x[e] * x[e];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rinv = 1.f / sqrtf(ss / static_cast<float>(D) + p.eps);
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = x[e] * rinv * to_f32(w[d0 + e]);
      }
      // RoPE (rotate_half): out[j] = x[j] cos - x[j+D/2] sin, out[j+D/2] = x[j+D/2] cos +
      // x[j] sin, angle pos * inv_freq[j mod D/2].
      const float pos = static_cast<float>(__ldg(p.positions + b));
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
        const int j = (d0 + e) & (D / 2 - 1);
        float s, c;
        sincosf(pos * __ldg(p.inv_freq + j), &s, &c);
        x[e] = upper ? x[e] * c + partner * s : x[e] * c - partner * s;
      }
    }

    To* dst;
    if (is_q) {
      dst = static_cast<To*>(p.q_out) + b * p.q_out_stride + kh * D;
    } else {
      const int64_t page = slot / p.page_size;
      const int64_t off = slot - page * p.page_size;
      char* pool = is_v ? p.v_pool : p.k_pool;
      dst = reinterpret_cast<To*>(pool) + ((page * p.hkv + kh) * p.page_size + off) * D;
    }
#pragma unroll
    for (int e = 0; e < E; ++e) dst[d0 + e] = from_f32<To>(x[e]);
  }
}

template <typename Ti, typename To>
int launch_prologue(const PrologueParams& p, int head_dim, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(p.batch) * (p.hq + 2 * p.hkv);
  int64_t blocks = (rows + 7) / 8;  // 8 warps per block
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const dim3 grid(static_cast<unsigned>(blocks));
  switch (head_dim) {
    case 64: return cuda_status(launch_kernel(decode_prologue_kernel<Ti, To, 2>, grid, dim3(256), 0, stream, p));
    case 128: return cuda_status(launch_kernel(decode_prologue_kernel<Ti, To, 4>, grid, dim3(256), 0, stream, p));
    case 256: return cuda_status(launch_kernel(decode_prologue_kernel<Ti, To, 8>, grid, dim3(256), 0, stream, p));
    default: return PI_ERR_UNSUPPORTED;
  }
}

template <typename Ti>
int dispatch_out(const PrologueParams& p, int head_dim, int pool_dtype, cudaStream_t stream) {
  switch (pool_dtype) {
    case PI_DTYPE_F32: return launch_prologue<Ti, float>(p, head_dim, stream);
    case PI_DTYPE_BF16: return launch_prologue<Ti, __nv_bfloat16>(p, head_dim, stream);
    case PI_DTYPE_F16: return launch_prologue<Ti, __half>(p, head_dim, stream);
    default: return PI_ERR_UNSUPPORTED;
  }
}

}  // namespace
}  // namespace pi

extern "C" int pi_decode_prologue(void* q_out, int64_t q_out_stride, void* k_pool, void* v_pool,
                                  const void* q_in, int64_t q_in_stride, const void* k_in,
                                  const void* v_in, int64_t kv_in_stride, int in_dtype,
                                  const void* q_norm_w, const void* k_norm_w, float eps,
                                  const float* inv_freq, const int64_t* positions,
                                  const int64_t* slot_mapping, int batch, int num_q_heads,
                                  int num_kv_heads, int head_dim, int page_size,
                                  int64_t num_slots, int pool_dtype, int* err,
                                  cudaStream_t stream) {
  using namespace pi;
  if (elem_bytes_of(in_dtype) == 0 || elem_bytes_of(pool_dtype) == 0) return PI_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return PI_ERR_UNSUPPORTED;
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || page_size <= 0 || num_slots < 0)
    return PI_ERR_BAD_SHAPE;
  if (q_out_stride < static_cast<int64_t>(num_q_heads) * head_dim ||
      q_in_stride < static_cast<int64_t>(num_q_heads) * head_dim ||
      kv_in_stride < static_cast<int64_t>(num_kv_heads) * head_dim)
    return PI_ERR_BAD_SHAPE;
  if (!(eps >= 0.f)) return PI_ERR_BAD_SHAPE;
  if (batch == 0) return PI_OK;
  if (!q_out || !k_pool || !v_pool || !q_in || !k_in || !v_in || !inv_freq || !positions ||
      !slot_mapping)
    return PI_ERR_NULL_POINTER;
  if ((q_norm_w == nullptr) != (k_norm_w == nullptr)) return PI_ERR_NULL_POINTER;
  if (!aligned(positions, 8) || !aligned(slot_mapping, 8) || !aligned(inv_freq, 4))
    return PI_ERR_MISALIGNED;
  PrologueParams p;
  p.q_out = q_out;
  p.k_pool = static_cast<char*>(k_pool);
  p.v_pool = static_cast<char*>(v_pool);
  p.q_in = q_in;
  p.k_in = k_in;
  p.v_in = v_in;
  p.q_norm_w = q_norm_w;
  p.k_norm_w = k_norm_w;
  p.inv_freq = inv_freq;
  p.positions = positions;
  p.slot_mapping = slot_mapping;
  p.q_out_stride = q_out_stride;
  p.q_in_stride = q_in_stride;
  p.kv_in_stride = kv_in_stride;
  p.num_slots = num_slots;
  p.eps = eps;
  p.batch = batch;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.page_size = page_size;
  p.err = err;
  switch (in_dtype) {
    case PI_DTYPE_F32: return dispatch_out<float>(p, head_dim, pool_dtype, stream);
    case PI_DTYPE_BF16: return dispatch_out<__nv_bfloat16>(p, head_dim, pool_dtype, stream);
    case PI_DTYPE_F16: return dispatch_out<__half>(p, head_dim, pool_dtype, stream);
    default: return PI_ERR_UNSUPPORTED;
  }
}
