// Paged prefill attention of one request (q_len new tokens), straight from the page pool.
//
//   out[i, hq] = softmax(scale * q[i, hq] . K[hq / G]^T) V[hq / G]  over keys j < lim(i),
//   lim(i) = min(kv_len, q_start + i + 1) when causal, kv_len otherwise.
//
// Replaces the prefill branch of the reference's _attn_paged
// (src/plastic_infer/exec/runner_paged.py:36-95): gather_paged_kv of the whole context,
// repeat_interleave of K/V over the G query heads of each KV head, then SDPA with
// is_causal (q_start_pos == 0, attention.py:151-190) or with a dense [q_len, kv_len] mask
// built for q_start_pos > 0. Here nothing is gathered or expanded: pages stream from
// the pool with TMA and the G heads of a KV head share every page.
//
// CTA = (block of T query tokens, KV head), 4 warps x 16 query rows = 64 rows, row
// rho = token * G + g (T = 64 / G). FA2 orientation on mma.sync m16n8k16: S = Q K^T with
// Q as the A operand held in registers for the whole KV loop, K^T fetched by ldmatrix
// from the swizzled page tile; P V with P taken straight from the S accumulators and V
// by ldmatrix.trans. Online softmax in base 2, fp32. The 4 warps consume one TMA ring of
// NS page stages (a "full" mbarrier per stage counts the TMA bytes). The CTA's page ids
// are staged in shared memory once; whichever warp finishes a stage last (a shared
// arrival counter) refills it at once, so no warp waits for another to issue loads.
// Every wait is bounded; a failing warp marks the CTA and thread 0 drains in-flight
// loads before the CTA exits.
#include <cudaTypedefs.h>

#include "pi_common.cuh"

namespace pi {
namespace attn {
// Cached 2-D tensor map over a physical pool [rows = P*Hkv*S, D] (paged_decode_attn.cu).
bool pool_tensor_map(CUtensorMap* out, const void* base, uint64_t rows, int D, int S, int dtype);
}  // namespace attn

namespace prefill {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kRows = 16 * kWarps;  // query rows per CTA
constexpr int kStages = 4;
constexpr int kIdCache = 2048;  // page ids staged in shared memory (32k tokens at S = 16)
constexpr unsigned kFull = 0xffffffffu;

template <int D, int S>
struct Cfg {
  static constexpr int kBoxes = D / 64;
  static constexpr int kBoxBytes = S * 128;
  static constexpr int kTileBytes = kBoxes * kBoxBytes;
  static constexpr int kStageBytes = 2 * kTileBytes;  // K + V
  static constexpr int kSub = S / 16;                 // 16-token sub-tiles per page
  static constexpr int kKK = D / 16;                  // QK k-steps
  static constexpr int kNT = D / 8;                   // PV n-tiles (O columns / 8)
};

// Byte offset of element (t, d) inside a swizzled [boxes][S][128 B] tile (128 B swizzle).
template <int S>
__device__ __forceinline__ uint32_t tile_off(int t, int d) {
  return static_cast<uint32_t>((d >> 6) * (S * 128) + t * 128 + ((((d & 63) >> 3) ^ (t & 7)) << 4));
}

struct PrefillParams {
  void* out;                  // [q_len, Hq, D], token stride out_tok_stride elements
  const void* q;              // [q_len, Hq, D], token stride q_tok_stride elements
  const int32_t* block_table; // [table_len] page ids of the request
  int64_t num_pages;
  int64_t q_tok_stride;
  int64_t out_tok_stride;
  int q_len, kv_len, q_start, causal;
  int hkv, group, tokens_per_cta, n_qblocks;
  float scale_log2;
  int* err;
};

template <typename T, int D, int S>
__global__ void __launch_bounds__(kThreads)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tmap_k,
                         const __grid_constant__ CUtensorMap tmap_v, const PrefillParams p) {
  using C = Cfg<D, S>;
  using Mma = MmaOp<T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(tiles + kStages * C::kStageBytes);
  __shared__ int s_failed;
  __shared__ int s_issued;           // pages issued so far (for the drain)
  __shared__ int s_arrived[kStages];  // warps done with the stage's current page
  __shared__ int s_tile[kIdCache];    // TMA tile row (page_id * Hkv + h) of page k

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int gid = lane >> 2;
  const int tig = lane & 3;
  const int G = p.group;
  const int h = blockIdx.x % p.hkv;
  // heaviest blocks (latest query tokens, most keys under a causal mask) first
  const int qb = p.n_qblocks - 1 - static_cast<int>(blockIdx.x / p.hkv);
  const int t0 = qb * p.tokens_per_cta;
  const int t_end = min(t0 + p.tokens_per_cta, p.q_len);
  // keys this CTA needs
  const int extent = p.causal ? min(p.kv_len, p.q_start + t_end) : p.kv_len;
  const int npages = (extent + S - 1) / S;

  // this lane's two rows (gid, gid + 8) of the warp's 16
  int tok[2], hq[2], lim[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int rho = warp * 16 + gid + 8 * i;
    tok[i] = t0 + rho / G;
    hq[i] = h * G + rho % G;
    const bool ok = tok[i] < p.q_len;
    lim[i] = !ok ? 0 : (p.causal ? min(p.kv_len, p.q_start + tok[i] + 1) : p.kv_len);
  }
  // smallest limit of the warp: pages wholly below it need no mask
  int wmin = min(lim[0], lim[1]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) wmin = min(wmin, __shfl_xor_sync(kFull, wmin, o));

  const uint32_t full0 = smem_u32(bars);
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(full0 + 8 * s, 1);
    fence_mbar_init();
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
    s_failed = 0;
    s_issued = 0;
  }
  if (tid < kStages) s_arrived[tid] = 0;

  // Programmatic launch: q, the pools and the block table may be the previous kernel's
  // output.
  pdl_wait();
  pdl_trigger();

  auto tile_of = [&](int k) -> int {
    int pid = __ldg(p.block_table + k);
    if (pid < 0 || static_cast<int64_t>(pid) >= p.num_pages) {
      record_error(p.err, PI_ERR_PAGE_RANGE);
      pid = 0;
    }
    return pid * p.hkv + h;
  };
  for (int i = tid; i < npages && i < kIdCache; i += kThreads) s_tile[i] = tile_of(i);
  __syncthreads();

  const uint32_t tiles_u32 = smem_u32(tiles);
  auto issue = [&](int k) {
    const int tile = k < kIdCache ? s_tile[k] : tile_of(k);
    const int stage = k % kStages;
    const uint32_t bar = full0 + 8 * stage;
    const uint32_t kdst = tiles_u32 + stage * C::kStageBytes;
    const uint32_t vdst = kdst + C::kTileBytes;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, C::kStageBytes);
#pragma unroll
    for (int j = 0; j < C::kBoxes; ++j) {
      tma_load_2d(kdst + j * C::kBoxBytes, &tmap_k, bar, 64 * j, tile * S);
      tma_load_2d(vdst + j * C::kBoxBytes, &tmap_v, bar, 64 * j, tile * S);
    }
  };
  if (tid == 0) {
    const int first = npages < kStages ? npages : kStages;
    for (int k = 0; k < first; ++k) issue(k);
    s_issued = first;
  }

  // Q rows as the MMA A operand for every k-step (rows past q_len are zero).
  uint32_t qa[C::kKK][4];
  {
    const T* q0 = static_cast<const T*>(p.q) + static_cast<int64_t>(tok[0]) * p.q_tok_stride + hq[0] * D;
    const T* q1 = static_cast<const T*>(p.q) + static_cast<int64_t>(tok[1]) * p.q_tok_stride + hq[1] * D;
    const bool v0 = tok[0] < p.q_len, v1 = tok[1] < p.q_len;
#pragma unroll
    for (int kk = 0; kk < C::kKK; ++kk) {
      const int d = 16 * kk + 2 * tig;
      qa[kk][0] = v0 ? __ldg(reinterpret_cast<const uint32_t*>(q0 + d)) : 0u;
      qa[kk][1] = v1 ? __ldg(reinterpret_cast<const uint32_t*>(q1 + d)) : 0u;
      qa[kk][2] = v0 ? __ldg(reinterpret_cast<const uint32_t*>(q0 + d + 8)) : 0u;
      qa[kk][3] = v1 ? __ldg(reinterpret_cast<const uint32_t*>(q1 + d + 8)) : 0u;
    }
  }

  // ldmatrix lane addressing: matrix mi = lane >> 3, row r = lane & 7
  const int mi = lane >> 3;
  const int mr = lane & 7;
  const int k_t = mr + 8 * (mi >> 1), k_d = 8 * (mi & 1);   // K^T: (tokens 0-7|8-15) x (d lo|hi)
  const int v_t = mr + 8 * (mi & 1), v_d = 8 * (mi >> 1);   // V (trans): (tokens lo|hi) x (d lo|hi)

  float o[C::kNT][4];
#pragma unroll
  for (int n = 0; n < C::kNT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  bool failed = false;

  for (int k = 0; k < npages; ++k) {
    const int stage = k % kStages;
    if (!mbar_wait_bounded(full0 + 8 * stage, static_cast<uint32_t>((k / kStages) & 1))) {
      if (lane == 0) record_error(p.err, PI_ERR_TIMEOUT);
      failed = true;
      break;
    }
    const uint32_t ktile = tiles_u32 + stage * C::kStageBytes;
    const uint32_t vtile = ktile + C::kTileBytes;
    const int j0 = k * S;
    const bool need_mask = j0 + S > wmin;
    const int vvalid = p.kv_len - j0;  // V rows at or past this are not context

    float s[C::kSub][2][4];
#pragma unroll
    for (int u = 0; u < C::kSub; ++u) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) s[u][nt][0] = s[u][nt][1] = s[u][nt][2] = s[u][nt][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < C::kKK; ++kk) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(ktile + tile_off<S>(16 * u + k_t, 16 * kk + k_d), b0, b1, b2, b3);
        Mma::run(s[u][0], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
        Mma::run(s[u][1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int j = j0 + 16 * u + 8 * nt + 2 * tig;
        if (need_mask) {
          s[u][nt][0] = j < lim[0] ? s[u][nt][0] * p.scale_log2 : -INFINITY;
          s[u][nt][1] = j + 1 < lim[0] ? s[u][nt][1] * p.scale_log2 : -INFINITY;
          s[u][nt][2] = j < lim[1] ? s[u][nt][2] * p.scale_log2 : -INFINITY;
          s[u][nt][3] = j + 1 < lim[1] ? s[u][nt][3] * p.scale_log2 : -INFINITY;
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) s[u][nt][c] *= p.scale_log2;
        }
      }
    }

    // online softmax, rows gid (elements 0, 1) and gid + 8 (elements 2, 3)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int u = 0; u < C::kSub; ++u)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        mx0 = fmaxf(mx0, fmaxf(s[u][nt][0], s[u][nt][1]));
        mx1 = fmaxf(mx1, fmaxf(s[u][nt][2], s[u][nt][3]));
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, 2));
    const float mn0 = fmaxf(m0, mx0);
    const float mn1 = fmaxf(m1, mx1);
    // a row with no key yet (mn = -inf) keeps alpha = 1 and p = 0
    const float al0 = mn0 == -INFINITY ? 1.f : fast_exp2(m0 - mn0);
    const float al1 = mn1 == -INFINITY ? 1.f : fast_exp2(m1 - mn1);
    const float sub0 = mn0 == -INFINITY ? 0.f : mn0;
    const float sub1 = mn1 == -INFINITY ? 0.f : mn1;
    m0 = mn0;
    m1 = mn1;
    uint32_t pa[C::kSub][4];
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int u = 0; u < C::kSub; ++u) {
      float e[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        e[nt][0] = fast_exp2(s[u][nt][0] - sub0);
        e[nt][1] = fast_exp2(s[u][nt][1] - sub0);
        e[nt][2] = fast_exp2(s[u][nt][2] - sub1);
        e[nt][3] = fast_exp2(s[u][nt][3] - sub1);
        ps0 += e[nt][0] + e[nt][1];
        ps1 += e[nt][2] + e[nt][3];
      }
      // the C fragments of the two 8-token n-tiles are the A fragment of P (16 tokens)
      pa[u][0] = Mma::pack(e[0][0], e[0][1]);
      pa[u][1] = Mma::pack(e[0][2], e[0][3]);
      pa[u][2] = Mma::pack(e[1][0], e[1][1]);
      pa[u][3] = Mma::pack(e[1][2], e[1][3]);
    }
    l0 = l0 * al0 + ps0;
    l1 = l1 * al1 + ps1;
#pragma unroll
    for (int n = 0; n < C::kNT; ++n) {
      o[n][0] *= al0;
      o[n][1] *= al0;
      o[n][2] *= al1;
      o[n][3] *= al1;
    }

    // O += P V. V rows past the context may hold anything (even NaN); P is 0 there but
    // 0 * NaN is not, so those rows are zeroed in the loaded fragments.
#pragma unroll
    for (int u = 0; u < C::kSub; ++u) {
      const int tb = 16 * u + 2 * tig;  // tokens tb, tb+1 (b0 / r2) and tb+8, tb+9 (b1 / r3)
      const bool tail = vvalid < 16 * u + 16;
      const uint32_t m_lo = (tb < vvalid ? 0x0000ffffu : 0u) | (tb + 1 < vvalid ? 0xffff0000u : 0u);
      const uint32_t m_hi = (tb + 8 < vvalid ? 0x0000ffffu : 0u) | (tb + 9 < vvalid ? 0xffff0000u : 0u);
#pragma unroll
      for (int jd = 0; jd < D / 16; ++jd) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(vtile + tile_off<S>(16 * u + v_t, 16 * jd + v_d), b0, b1, b2, b3);
        if (tail) {
          b0 &= m_lo;
          b1 &= m_hi;
          b2 &= m_lo;
          b3 &= m_hi;
        }
        Mma::run(o[2 * jd], pa[u][0], pa[u][1], pa[u][2], pa[u][3], b0, b1);
        Mma::run(o[2 * jd + 1], pa[u][0], pa[u][1], pa[u][2], pa[u][3], b2, b3);
      }
    }

    // The last warp done with this stage refills it with page k + NS: this warp's reads of
    // the stage precede its count (warp barrier + CTA-scope release); the last counter
    // acquires every warp's, then hands the stage to the async proxy.
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&s_arrived[stage], 1) == kWarps - 1) {
        __threadfence_block();
        s_arrived[stage] = 0;
        if (k + kStages < npages) {
          issue(k + kStages);
          atomicAdd(&s_issued, 1);
        }
      }
    }
  }
  if (failed) atomicOr(&s_failed, 1);

  // row sums over the 4 lanes of a row, then normalise and store (rows past q_len skipped)
  l0 += __shfl_xor_sync(kFull, l0, 1);
  l0 += __shfl_xor_sync(kFull, l0, 2);
  l1 += __shfl_xor_sync(kFull, l1, 1);
  l1 += __shfl_xor_sync(kFull, l1, 2);
  const float i0 = l0 > 0.f ? 1.f / l0 : 0.f;
  const float i1 = l1 > 0.f ? 1.f / l1 : 0.f;
  T* out0 = static_cast<T*>(p.out) + static_cast<int64_t>(tok[0]) * p.out_tok_stride + hq[0] * D;
  T* out1 = static_cast<T*>(p.out) + static_cast<int64_t>(tok[1]) * p.out_tok_stride + hq[1] * D;
#pragma unroll
  for (int n = 0; n < C::kNT; ++n) {
    const int d = 8 * n + 2 * tig;
    if (tok[0] < p.q_len)
      *reinterpret_cast<uint32_t*>(out0 + d) = Mma::pack(o[n][0] * i0, o[n][1] * i0);
    if (tok[1] < p.q_len)
      *reinterpret_cast<uint32_t*>(out1 + d) = Mma::pack(o[n][2] * i1, o[n][3] * i1);
  }

  // Before shared memory is released: on any failure, wait (bounded) for every load in
  // flight; the last kStages issued pages are the only ones that can still be landing.
  __syncthreads();
  if (tid == 0 && s_failed) {
    const int issued = s_issued;
    for (int j = issued > kStages ? issued - kStages : 0; j < issued; ++j)
      mbar_wait_bounded(full0 + 8 * (j % kStages), static_cast<uint32_t>((j / kStages) & 1));
  }
}

template <typename T, int D, int S>
int launch(const PrefillParams& p, const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t stream) {
  using C = Cfg<D, S>;
  constexpr size_t smem = 1024 + static_cast<size_t>(kStages) * C::kStageBytes + kStages * 8;
  auto kern = paged_prefill_kernel<T, D, S>;
  static bool configured[64] = {};  // per device: the dynamic shared memory limit is set
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return PI_ERR_CUDA;
  bool& done = configured[dev];
  if (!done) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return PI_ERR_CUDA;
    done = true;
  }
  const dim3 grid(static_cast<unsigned>(p.n_qblocks) * static_cast<unsigned>(p.hkv));
  return cuda_status(launch_kernel(kern, grid, dim3(kThreads), smem, stream, tk, tv, p));
}

}  // namespace
}  // namespace prefill
}  // namespace pi

extern "C" int pi_paged_prefill_attn(void* out, const void* q, const void* k_pool,
                                     const void* v_pool, const int32_t* block_table,
                                     int64_t table_len, int q_len, int kv_len, int q_start,
                                     int causal, int num_q_heads, int num_kv_heads, int head_dim,
                                     int page_size, int64_t num_pages, float scale, int dtype,
                                     int64_t q_tok_stride, int64_t out_tok_stride, int* err,
                                     cudaStream_t stream) {
  using namespace pi;
  if (dtype != PI_DTYPE_BF16 && dtype != PI_DTYPE_F16) return PI_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return PI_ERR_UNSUPPORTED;
  if (page_size != 16 && page_size != 32) return PI_ERR_UNSUPPORTED;
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads) return PI_ERR_BAD_SHAPE;
  const int G = num_q_heads / num_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8 && G != 16) return PI_ERR_UNSUPPORTED;
  if (q_len < 0 || kv_len < 0 || q_start < 0 || num_pages <= 0 || table_len < 0)
    return PI_ERR_BAD_SHAPE;
  if (static_cast<int64_t>(kv_len) > table_len * page_size) return PI_ERR_BAD_SHAPE;
  if (q_tok_stride < static_cast<int64_t>(num_q_heads) * head_dim ||
      out_tok_stride < static_cast<int64_t>(num_q_heads) * head_dim)
    return PI_ERR_BAD_SHAPE;
  if (static_cast<int64_t>(num_pages) * num_kv_heads * page_size > (int64_t{1} << 31))
    return PI_ERR_BAD_SHAPE;  // TMA row coordinate is a 32-bit int
  if (q_len == 0) return PI_OK;
  if (!out || !q || !k_pool || !v_pool || (kv_len > 0 && !block_table)) return PI_ERR_NULL_POINTER;
  if (!aligned(q, 4) || !aligned(out, 4) || (q_tok_stride % 2) || (out_tok_stride % 2) ||
      !aligned(k_pool, 16) || !aligned(v_pool, 16))
    return PI_ERR_MISALIGNED;
  const uint64_t rows = static_cast<uint64_t>(num_pages) * num_kv_heads * page_size;
  CUtensorMap tk, tv;
  if (!attn::pool_tensor_map(&tk, k_pool, rows, head_dim, page_size, dtype) ||
      !attn::pool_tensor_map(&tv, v_pool, rows, head_dim, page_size, dtype))
    return PI_ERR_CUDA;
  prefill::PrefillParams p;
  p.out = out;
  p.q = q;
  p.block_table = block_table;
  p.num_pages = num_pages;
  p.q_tok_stride = q_tok_stride;
  p.out_tok_stride = out_tok_stride;
  p.q_len = q_len;
  p.kv_len = kv_len;
  p.q_start = q_start;
  p.causal = causal ? 1 : 0;
  p.hkv = num_kv_heads;
  p.group = G;
  p.tokens_per_cta = prefill::kRows / G;
  p.n_qblocks = (q_len + p.tokens_per_cta - 1) / p.tokens_per_cta;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = err;
#define PI_PREFILL(T, D, S)                                  \
  if (head_dim == D && page_size == S)                       \
    return prefill::launch<T, D, S>(p, tk, tv, stream);
  if (dtype == PI_DTYPE_BF16) {
    PI_PREFILL(__nv_bfloat16, 64, 16)
    PI_PREFILL(__nv_bfloat16, 128, 16)
    PI_PREFILL(__nv_bfloat16, 64, 32)
    PI_PREFILL(__nv_bfloat16, 128, 32)
  } else {
    PI_PREFILL(__half, 64, 16)
    PI_PREFILL(__half, 128, 16)
    PI_PREFILL(__half, 64, 32)
    PI_PREFILL(__half, 128, 32)
  }
#undef PI_PREFILL
  return PI_ERR_UNSUPPORTED;
}
