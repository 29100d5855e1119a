// pi_host_stream_attn: attention over a KV sequence split between host-resident chunks
// and a device-resident tail, read in place.
//
// Replaces host_stream_attention_v1 (src/plastic_infer/exec/attention.py:193-250), the
// reference's long-sequence HOST_STREAM primitive: it concatenates the host chunks
// ([H_kv, D, C] each, oldest first) and the resident tail ([1, R, H_kv, D]) into one
// contiguous buffer, repeats each KV head G times and runs SDPA with the offset causal
// mask (key j visible to query i iff j <= q_start + i). Its docstring names the swap this
// file makes: a flash-incremental kernel that reads the host chunks without
// materialising them.
//
// Design (B200, host link bound):
// - The KV sequence is a list of spans: (k, v, len, strides). A span's memory is either
//   device memory or page-locked host memory read through the device's mapped view of
//   it, so host chunks cross the link exactly once and are never staged.
// - Grid (split, row block, KV head). A CTA owns one KV head, up to kRB query rows of it
//   (row = query token i * G + head offset g, so the G heads of a KV head share every
//   K/V block) and a contiguous token range. Splits over tokens give the link enough
//   loads in flight: one decode request of 32k tokens becomes ~600 CTAs.
// - Per 32-token block, the 4 warps load K and V rows with 16-byte loads (token-major
//   spans) or strided element loads (any other layout) into fp32 shared tiles; each warp
//   then runs an online base-2 softmax for its rows, one lane per token for the scores
//   and one lane per column for P.V.
// - Splits leave (m, l, O) partials; a second kernel merges them per row. With one split
//   the first kernel writes the output directly.
// The arithmetic is SIMT fp32: at the link's ~55 GB/s a decode step needs ~0.2 TFLOP/s.
#include "pi_common.cuh"

#include <algorithm>
#include <type_traits>

namespace pi {
namespace hs {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kBT = 32;                  // tokens per block (one per lane for the scores)
constexpr int kRB = 16;                  // query rows per CTA
constexpr int kRPW = kRB / kWarps;       // rows per warp
constexpr int kCtasPerSm = 3;            // CTAs resident per SM (170 registers a thread)

struct Span {
  const void* k;
  const void* v;
  int64_t start;  // first token of the span in the sequence
  int64_t head_stride;
  int64_t tok_stride;
  int64_t dim_stride;
  int vec;        // 16-byte loads along head_dim are valid for this span
  int pad;
};

struct Params {
  void* out;
  const void* q;
  float* ws_o;   // [hkv][nrb][kRB][nsplit][D] partial O
  float* ws_ml;  // [hkv][nrb][kRB][nsplit][2] partial (m, l)
  int64_t q_tok_stride;
  int64_t out_tok_stride;
  int64_t q_start;
  int64_t kv_len;
  int64_t tokens_per_split;
  int q_len;
  int hkv;
  int group;
  int head_dim;
  int nsplit;
  int nrb;
  int num_spans;
  int causal;
  float scale_log2;
  int* err;
  Span spans[PI_HS_MAX_SPANS];
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One element of T, held in the low bits of `b`, as fp32.
template <typename T>
__device__ __forceinline__ float bits_to_f32(uint32_t b) {
  if constexpr (sizeof(T) == 4) {
    return __uint_as_float(b);
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return __uint_as_float(b << 16);
  } else {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(b)));
  }
}

// 16 bytes holding 16 / sizeof(T) consecutive elements of T as fp32 into dst.
template <typename T>
__device__ __forceinline__ void cvt16(const uint4 u, float* dst) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(dst) = make_float4(__uint_as_float(u.x), __uint_as_float(u.y),
                                                  __uint_as_float(u.z), __uint_as_float(u.w));
  } else {
    *reinterpret_cast<float4*>(dst) =
        make_float4(bits_to_f32<T>(u.x & 0xffffu), bits_to_f32<T>(u.x >> 16),
                    bits_to_f32<T>(u.y & 0xffffu), bits_to_f32<T>(u.y >> 16));
    *reinterpret_cast<float4*>(dst + 4) =
        make_float4(bits_to_f32<T>(u.z & 0xffffu), bits_to_f32<T>(u.z >> 16),
                    bits_to_f32<T>(u.w & 0xffffu), bits_to_f32<T>(u.w >> 16));
  }
}

// 16 / sizeof(T) elements of T at p, p + stride, ... packed like a 16-byte vector.
template <typename T>
__device__ __forceinline__ uint4 gather16(const T* p, int64_t stride) {
  if constexpr (sizeof(T) == 4) {
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p);
    return make_uint4(q[0], q[stride], q[2 * stride], q[3 * stride]);
  } else {
    const unsigned short* q = reinterpret_cast<const unsigned short*>(p);
    auto pair = [&](int i) {
      return static_cast<uint32_t>(q[2 * i * stride]) | (static_cast<uint32_t>(q[(2 * i + 1) * stride]) << 16);
    };
    return make_uint4(pair(0), pair(1), pair(2), pair(3));
  }
}

// Shared memory: K and V tiles [kBT][D + 4] fp32 (the pad keeps the per-lane row reads
// of the score loop free of bank conflicts) and the scaled query rows [kRB][D].
inline size_t smem_bytes(int D) {
  return static_cast<size_t>(2 * kBT * (D + 4) + kRB * D) * 4;
}

// kDL = columns per lane in P.V (D <= 32 * kDL).
template <typename T, int kDL>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) host_stream_attn_kernel(const __grid_constant__ Params p) {
  extern __shared__ float sm[];
  const int D = p.head_dim;
  const int DP = D + 4;
  float* ks = sm;
  float* vs = ks + kBT * DP;
  float* qs = vs + kBT * DP;

  const int split = blockIdx.x;
  const int rb = blockIdx.y;
  const int h = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = p.group;
  const int R = p.q_len * G;
  const int r0 = rb * kRB;
  const int nr = min(kRB, R - r0);
  constexpr int kEsz = static_cast<int>(sizeof(T));
  constexpr int kEpv = 16 / kEsz;          // elements per 16-byte vector
  const int V = D / kEpv;                  // vectors per row (D is a multiple of kEpv)

  pdl_trigger();
  pdl_wait();

  // query rows, pre-scaled into the base-2 softmax domain
  for (int idx = tid; idx < nr * D; idx += kThreads) {
    const int rr = idx / D;
    const int d = idx - rr * D;
    const int r = r0 + rr;
    const int i = r / G;
    const int g = r - i * G;
    qs[rr * D + d] = to_f32(static_cast<const T*>(p.q)[i * p.q_tok_stride + (h * G + g) * D + d]) *
                     p.scale_log2;
  }
  __syncthreads();

  const int64_t t_begin = static_cast<int64_t>(split) * p.tokens_per_split;
  const int64_t t_end = min(p.kv_len, t_begin + p.tokens_per_split);

  float o[kRPW][kDL];
  float m[kRPW], l[kRPW];
#pragma unroll
  for (int j = 0; j < kRPW; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.f;
#pragma unroll
    for (int e = 0; e < kDL; ++e) o[j][e] = 0.f;
  }

  // The span table lives in the parameter block, read through the constant cache,
  // which serves one address per warp-wide load at full speed and serialises
  // divergent ones. So every span read below has one index for the whole warp: a
  // binary search for the range's first span, then the current span's descriptor held
  // in registers and advanced in order. Only a token past the current span inside a
  // block (a span shorter than a block) takes the per-lane path.
  auto span_end = [&](int s) { return s + 1 < p.num_spans ? p.spans[s + 1].start : p.kv_len; };
  int sb = 0;
  {
    int lo = 0, hi = p.num_spans - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.spans[mid].start <= t_begin) lo = mid; else hi = mid - 1;
    }
    sb = lo;
  }
  const T* ck;
  const T* cv;
  int64_t c_start, c_end, c_hs, c_ts, c_ds;
  bool c_vec;
  auto load_cur = [&]() {
    const Span& sp = p.spans[sb];
    ck = static_cast<const T*>(sp.k);
    cv = static_cast<const T*>(sp.v);
    c_start = sp.start;
    c_end = span_end(sb);
    c_hs = sp.head_stride;
    c_ts = sp.tok_stride;
    c_ds = sp.dim_stride;
    c_vec = sp.vec != 0;
  };
  load_cur();

  // ---- loads, register-staged one block ahead: lane c of warp w loads 16-byte vector
  // c % V of tokens w + 4 (c / V) of the block, so every load of a block is issued
  // before any of them is used and the next block's loads fly during this block's math.
  // A span that does not allow 16-byte loads is read element by element into the same
  // raw vector.
  constexpr int kIt = (8 * 32 * kDL / kEpv + 31) / 32 < 8 ? (8 * 32 * kDL / kEpv + 31) / 32 : 8;
  uint4 rk[kIt], rv[kIt];
  auto fetch = [&](int64_t t0, int c, uint4& ko, uint4& vo) {
    const int tt = warp + kWarps * (c / V);
    const int vi = c - (c / V) * V;
    const int64_t pos = t0 + tt;
    const T* kb = ck;
    const T* vb = cv;
    int64_t start = c_start, hs = c_hs, ts = c_ts, ds = c_ds;
    bool vec = c_vec;
    if (pos >= c_end) {  // a later span inside this block
      int s = sb + 1;
      while (span_end(s) <= pos) ++s;
      const Span& sp = p.spans[s];
      kb = static_cast<const T*>(sp.k);
      vb = static_cast<const T*>(sp.v);
      start = sp.start;
      hs = sp.head_stride;
      ts = sp.tok_stride;
      ds = sp.dim_stride;
      vec = sp.vec != 0;
    }
    const int64_t off = h * hs + (pos - start) * ts + static_cast<int64_t>(vi) * kEpv * ds;
    if (vec) {
      ko = *reinterpret_cast<const uint4*>(kb + off);
      vo = *reinterpret_cast<const uint4*>(vb + off);
    } else {
      ko = gather16<T>(kb + off, ds);
      vo = gather16<T>(vb + off, ds);
    }
  };
  auto issue = [&](int64_t t0) {
    while (t0 >= c_end) {  // warp-uniform: move the current span to the block's first token
      ++sb;
      load_cur();
    }
    const int nt = static_cast<int>(min(static_cast<int64_t>(kBT), t_end - t0));
#pragma unroll
    for (int it = 0; it < kIt; ++it) {
      const int c = lane + 32 * it;
      if (c < (kBT / kWarps) * V && warp + kWarps * (c / V) < nt) fetch(t0, c, rk[it], rv[it]);
    }
  };
  auto put = [&](int c, const uint4& ko, const uint4& vo, bool valid) {
    const int tt = warp + kWarps * (c / V);
    const int vi = c - (c / V) * V;
    float* kd = ks + tt * DP + vi * kEpv;
    float* vd = vs + tt * DP + vi * kEpv;
    if (valid) {
      cvt16<T>(ko, kd);
      cvt16<T>(vo, vd);
    } else {
#pragma unroll
      for (int e = 0; e < kEpv; ++e) kd[e] = vd[e] = 0.f;
    }
  };
  // staged vectors -> fp32 tiles (and, past what the registers stage, direct loads)
  auto store = [&](int64_t t0, int nt) {
#pragma unroll
    for (int it = 0; it < kIt; ++it) {
      const int c = lane + 32 * it;
      if (c < (kBT / kWarps) * V) put(c, rk[it], rv[it], warp + kWarps * (c / V) < nt);
    }
    for (int c = lane + 32 * kIt; c < (kBT / kWarps) * V; c += 32) {
      uint4 ko, vo;
      const bool valid = warp + kWarps * (c / V) < nt;
      if (valid) fetch(t0, c, ko, vo);
      put(c, ko, vo, valid);
    }
  };

  if (t_begin < t_end) issue(t_begin);
  for (int64_t t0 = t_begin; t0 < t_end; t0 += kBT) {
    const int nt = static_cast<int>(min(static_cast<int64_t>(kBT), t_end - t0));
    store(t0, nt);
    __syncthreads();
    if (t0 + kBT < t_end) issue(t0 + kBT);
    // ---- scores and online softmax: lane = token for S, lane = column for P.V
#pragma unroll
    for (int j = 0; j < kRPW; ++j) {
      const int rr = warp + j * kWarps;
      if (rr >= nr) break;
      // causal: row r (query token r / G) sees keys up to q_start + r / G
      const int64_t lim = p.causal ? p.q_start + (r0 + rr) / G : INT64_MAX;
      float s = -INFINITY;
      if (lane < nt && t0 + lane <= lim) {
        const float* kr = ks + lane * DP;
        const float* qr = qs + rr * D;
        float a0 = 0.f, a1 = 0.f;
#pragma unroll 4
        for (int d = 0; d < D; d += 8) {
          const float4 k0 = *reinterpret_cast<const float4*>(kr + d);
          const float4 q0 = *reinterpret_cast<const float4*>(qr + d);
          a0 += k0.x * q0.x + k0.y * q0.y + k0.z * q0.z + k0.w * q0.w;
          if (d + 4 < D) {
            const float4 k1 = *reinterpret_cast<const float4*>(kr + d + 4);
            const float4 q1 = *reinterpret_cast<const float4*>(qr + d + 4);
            a1 += k1.x * q1.x + k1.y * q1.y + k1.z * q1.z + k1.w * q1.w;
          }
        }
        s = a0 + a1;
      }
      const float mx = warp_max(s);
      if (mx == -INFINITY) continue;  // nothing visible to this row in the block
      const float mn = fmaxf(m[j], mx);
      const float a = m[j] == -INFINITY ? 0.f : fast_exp2(m[j] - mn);
      const float pe = s == -INFINITY ? 0.f : fast_exp2(s - mn);
      l[j] = l[j] * a + warp_sum(pe);
      m[j] = mn;
#pragma unroll
      for (int e = 0; e < kDL; ++e) o[j][e] *= a;
      for (int t = 0; t < nt; ++t) {
        const float pt = __shfl_sync(0xffffffffu, pe, t);
        const float* vr = vs + t * DP;
#pragma unroll
        for (int e = 0; e < kDL; ++e) {
          const int d = lane + 32 * e;
          if (d < D) o[j][e] += pt * vr[d];
        }
      }
    }
    __syncthreads();
  }

  // ---- results: the output rows (one split) or this split's partials
#pragma unroll
  for (int j = 0; j < kRPW; ++j) {
    const int rr = warp + j * kWarps;
    if (rr >= nr) break;
    const int r = r0 + rr;
    if (p.nsplit == 1) {
      const int i = r / G;
      const int g = r - i * G;
      T* orow = static_cast<T*>(p.out) + i * p.out_tok_stride + (h * G + g) * D;
      const float inv = l[j] > 0.f ? 1.f / l[j] : 0.f;
#pragma unroll
      for (int e = 0; e < kDL; ++e) {
        const int d = lane + 32 * e;
        if (d < D) orow[d] = from_f32<T>(o[j][e] * inv);
      }
    } else {
      const int64_t idx = ((static_cast<int64_t>(h) * p.nrb + rb) * kRB + rr) * p.nsplit + split;
      float* wo = p.ws_o + idx * D;
#pragma unroll
      for (int e = 0; e < kDL; ++e) {
        const int d = lane + 32 * e;
        if (d < D) wo[d] = o[j][e];
      }
      if (lane == 0) {
        p.ws_ml[idx * 2] = m[j];
        p.ws_ml[idx * 2 + 1] = l[j];
      }
    }
  }
}

// Merge the splits of every row: one warp per (KV head, row).
template <typename T>
__global__ void __launch_bounds__(kThreads) host_stream_combine_kernel(const __grid_constant__ Params p) {
  pdl_trigger();
  pdl_wait();
  const int D = p.head_dim;
  const int G = p.group;
  const int R = p.q_len * G;
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (wid >= static_cast<int64_t>(p.hkv) * R) return;
  const int h = static_cast<int>(wid / R);
  const int r = static_cast<int>(wid - static_cast<int64_t>(h) * R);
  const int rb = r / kRB;
  const int rr = r - rb * kRB;
  const int64_t base = ((static_cast<int64_t>(h) * p.nrb + rb) * kRB + rr) * p.nsplit;
  float M = -INFINITY;
  for (int s = lane; s < p.nsplit; s += 32) M = fmaxf(M, p.ws_ml[(base + s) * 2]);
  M = warp_max(M);
  const int i = r / G;
  const int g = r - i * G;
  T* orow = static_cast<T*>(p.out) + i * p.out_tok_stride + (h * G + g) * D;
  float L = 0.f;
  for (int s = lane; s < p.nsplit; s += 32) {
    const float ms = p.ws_ml[(base + s) * 2];
    if (ms != -INFINITY) L += fast_exp2(ms - M) * p.ws_ml[(base + s) * 2 + 1];
  }
  L = warp_sum(L);
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int d = lane; d < D; d += 32) {
    float acc = 0.f;
#pragma unroll 4
    for (int s = 0; s < p.nsplit; ++s) {
      const float ms = p.ws_ml[(base + s) * 2];
      if (ms != -INFINITY) acc += fast_exp2(ms - M) * p.ws_o[(base + s) * D + d];
    }
    orow[d] = from_f32<T>(M == -INFINITY ? 0.f : acc * inv);
  }
}

// Split plan shared by the workspace query and the launch.
struct Plan {
  int nrb;
  int nsplit;
  int64_t tokens_per_split;
};

inline Plan make_plan(int q_len, int G, int hkv, int64_t kv_len) {
  Plan pl;
  const int64_t R = static_cast<int64_t>(q_len) * G;
  pl.nrb = static_cast<int>((R + kRB - 1) / kRB);
  const int64_t blocks = std::max<int64_t>(1, (kv_len + kBT - 1) / kBT);
  const int64_t units = static_cast<int64_t>(hkv) * pl.nrb;
  const int64_t target = static_cast<int64_t>(device_sm_count()) * kCtasPerSm;
  int64_t ns = std::max<int64_t>(1, (target + units - 1) / units);
  ns = std::min<int64_t>(ns, blocks);
  ns = std::min<int64_t>(ns, 65535);
  const int64_t bps = (blocks + ns - 1) / ns;  // blocks per split
  pl.tokens_per_split = bps * kBT;
  pl.nsplit = static_cast<int>((blocks + bps - 1) / bps);
  return pl;
}

inline size_t workspace_bytes(const Plan& pl, int hkv, int D) {
  if (pl.nsplit <= 1) return 0;
  const size_t rows = static_cast<size_t>(hkv) * pl.nrb * kRB * pl.nsplit;
  return ((rows * 2 * 4 + 255) & ~static_cast<size_t>(255)) + rows * D * 4;
}

template <typename T, int kDL>
int launch(const Params& p, size_t smem, cudaStream_t stream) {
  auto kern = host_stream_attn_kernel<T, kDL>;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return PI_ERR_CUDA;
  }
  cudaError_t e = launch_kernel(kern, dim3(p.nsplit, p.nrb, p.hkv), dim3(kThreads), smem, stream, p);
  if (e != cudaSuccess) return PI_ERR_CUDA;
  if (p.nsplit > 1) {
    const int64_t rows = static_cast<int64_t>(p.hkv) * p.q_len * p.group;
    const unsigned blocks = static_cast<unsigned>((rows + kWarps - 1) / kWarps);
    e = launch_kernel(host_stream_combine_kernel<T>, dim3(blocks), dim3(kThreads), 0, stream, p);
    if (e != cudaSuccess) return PI_ERR_CUDA;
  }
  return PI_OK;
}

template <typename T>
int dispatch(const Params& p, size_t smem, cudaStream_t stream) {
  const int D = p.head_dim;
  if (D <= 32) return launch<T, 1>(p, smem, stream);
  if (D <= 64) return launch<T, 2>(p, smem, stream);
  if (D <= 128) return launch<T, 4>(p, smem, stream);
  return launch<T, 8>(p, smem, stream);
}

// Device address of `ptr` for a kernel on the current device: device memory as is,
// page-locked host memory through its mapped device alias. Pageable memory has none.
inline bool device_alias(const void* ptr, const void** out) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
    *out = ptr;
    return true;
  }
  if (a.type == cudaMemoryTypeHost && a.devicePointer != nullptr) {
    *out = a.devicePointer;
    return true;
  }
  return false;
}

// Whether the current device reads page-locked host memory at its host address (the
// pinned allocations of cudaHostAlloc always; registered ones per this attribute).
inline bool host_pointers_usable() {
  static int cached[64] = {};  // 0 unknown, 1 yes, 2 no
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (cached[dev] == 0) {
    int v = 0;
    const bool ok = cudaDeviceGetAttribute(&v, cudaDevAttrCanUseHostPointerForRegisteredMem, dev) ==
                    cudaSuccess;
    cached[dev] = ok && v ? 1 : 2;
  }
  return cached[dev] == 1;
}

}  // namespace hs
}  // namespace pi

extern "C" size_t pi_host_stream_attn_workspace_size(int q_len, int num_q_heads, int num_kv_heads,
                                                     int head_dim, int64_t kv_len) {
  using namespace pi::hs;
  if (q_len <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads ||
      head_dim <= 0 || kv_len < 0)
    return 0;
  const Plan pl = make_plan(q_len, num_q_heads / num_kv_heads, num_kv_heads, kv_len);
  return workspace_bytes(pl, num_kv_heads, head_dim);
}

extern "C" int pi_host_stream_attn(void* out, const void* q, int64_t q_tok_stride,
                                   int64_t out_tok_stride, const pi_kv_span_t* spans,
                                   int num_spans, int q_len, int64_t q_start, int causal,
                                   int num_q_heads, int num_kv_heads, int head_dim, float scale,
                                   int dtype, void* workspace, size_t workspace_bytes_given,
                                   int flags, int* err, cudaStream_t stream) {
  using namespace pi;
  using namespace pi::hs;
  const int esz = elem_bytes_of(dtype);
  if (esz == 0) return PI_ERR_UNSUPPORTED;
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads) return PI_ERR_BAD_SHAPE;
  if (head_dim <= 0 || head_dim > 256 || head_dim % 8) return PI_ERR_UNSUPPORTED;
  if (q_len < 0 || q_start < 0 || num_spans < 0) return PI_ERR_BAD_SHAPE;
  if (num_spans > PI_HS_MAX_SPANS) return PI_ERR_UNSUPPORTED;
  if (q_tok_stride < static_cast<int64_t>(num_q_heads) * head_dim ||
      out_tok_stride < static_cast<int64_t>(num_q_heads) * head_dim)
    return PI_ERR_BAD_SHAPE;
  if (q_len == 0) return PI_OK;
  if (!out || !q || (num_spans > 0 && !spans)) return PI_ERR_NULL_POINTER;
  if (!aligned(q, esz) || !aligned(out, esz)) return PI_ERR_MISALIGNED;

  // ~29 KB: one block per calling thread, not on its stack (the launch copies it)
  static thread_local Params tl_params;
  Params* p = &tl_params;
  p->out = out;
  p->q = q;
  p->q_tok_stride = q_tok_stride;
  p->out_tok_stride = out_tok_stride;
  p->q_start = q_start;
  p->q_len = q_len;
  p->hkv = num_kv_heads;
  p->group = num_q_heads / num_kv_heads;
  p->head_dim = head_dim;
  p->causal = causal ? 1 : 0;
  p->scale_log2 = scale * 1.4426950408889634f;
  p->err = err;
  // Spans: empty ones are dropped; the rest get their start and device alias.
  const bool checked = (flags & PI_HS_SPANS_CHECKED) != 0 && host_pointers_usable();
  int64_t kv_len = 0;
  int n = 0;
  for (int i = 0; i < num_spans; ++i) {
    const pi_kv_span_t& s = spans[i];
    if (s.len < 0 || s.head_stride < 0 || s.tok_stride < 0 || s.dim_stride < 0) return PI_ERR_BAD_SHAPE;
    if (s.len == 0) continue;
    if (!s.k || !s.v) return PI_ERR_NULL_POINTER;
    if (!aligned(s.k, esz) || !aligned(s.v, esz)) return PI_ERR_MISALIGNED;
    Span& d = p->spans[n++];
    if (checked) {
      d.k = s.k;
      d.v = s.v;
    } else if (!device_alias(s.k, &d.k) || !device_alias(s.v, &d.v)) {
      return PI_ERR_UNSUPPORTED;
    }
    d.start = kv_len;
    d.head_stride = s.head_stride;
    d.tok_stride = s.tok_stride;
    d.dim_stride = s.dim_stride;
    d.vec = s.dim_stride == 1 && aligned(d.k, 16) && aligned(d.v, 16) &&
            (s.head_stride * esz) % 16 == 0 && (s.tok_stride * esz) % 16 == 0;
    d.pad = 0;
    kv_len += s.len;
  }
  if (n == 0) {  // no keys at all: one split, every row reads nothing and writes zeros
    Span& d = p->spans[n++];
    d = Span{q, q, 0, 0, 0, 1, 0, 0};
  }
  p->num_spans = n;
  p->kv_len = kv_len;
  const Plan pl = make_plan(q_len, p->group, num_kv_heads, kv_len);
  if (pl.nrb > 65535) return PI_ERR_UNSUPPORTED;  // grid y
  p->nrb = pl.nrb;
  p->nsplit = pl.nsplit;
  p->tokens_per_split = pl.tokens_per_split;
  const size_t need = workspace_bytes(pl, num_kv_heads, head_dim);
  if (need > 0) {
    if (!workspace || workspace_bytes_given < need) return PI_ERR_WORKSPACE;
    if (!aligned(workspace, 256)) return PI_ERR_MISALIGNED;
    const size_t rows = static_cast<size_t>(num_kv_heads) * pl.nrb * kRB * pl.nsplit;
    p->ws_ml = static_cast<float*>(workspace);
    p->ws_o = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                       ((rows * 2 * 4 + 255) & ~static_cast<size_t>(255)));
  } else {
    p->ws_ml = nullptr;
    p->ws_o = nullptr;
  }
  const size_t smem = smem_bytes(head_dim);
  if (smem > 227 * 1024) return PI_ERR_UNSUPPORTED;
  if (dtype == PI_DTYPE_F32) return dispatch<float>(*p, smem, stream);
  if (dtype == PI_DTYPE_BF16) return dispatch<__nv_bfloat16>(*p, smem, stream);
  return dispatch<__half>(*p, smem, stream);
}
