// Paged prefill attention on the 5th-generation tensor cores (tcgen05, TMEM accumulators).
//
// Same operation and arguments as pi_paged_prefill_attn (paged_prefill_attn.cu), which
// replaces the prefill branch of the reference's _attn_paged
// (src/plastic_infer/exec/runner_paged.py:36-95):
//   out[i, hq] = softmax(scale * q[i, hq] . K[hq / G]^T) V[hq / G]  over keys j < lim(i),
//   lim(i) = min(kv_len, q_start + i + 1) when causal, kv_len otherwise.
//
// CTA = (block of 128 / G query tokens, KV head): 128 query rows, row r = token * G + g,
// one row per thread and per TMEM lane. The context streams in tiles of 64 keys (64 / S
// pages by TMA): K and V each through a 2-slot ring. Per tile:
//   1. one thread issues S = Q K^T: tcgen05.mma kind::f16, M = 128, N = 64, K = 16 steps,
//      A = Q and B = the K tile, both K-major with the 128-byte swizzle; S lands in TMEM
//      columns [0, 64);
//   2. every thread reads its row of S (tcgen05.ld 32x32b), masks it and runs the online
//      softmax in base 2; P goes to shared memory, swizzled K-major. The running maximum
//      moves only when a row's new maximum exceeds it by more than 2^8, so P <= 256 and O
//      (TMEM) is rescaled on those rare tiles only; the stale maximum cancels in O / l;
//   3. one thread issues O += P V: A = P (K-major), B = the V tile, MN-major (its rows are
//      head_dim-contiguous per key).
// K(j + 2) and V(j + 1) load while tile j computes; thread 0 reads the page ids of a tile
// one iteration before it issues the tile's loads. The CTA needs 113 KB of shared memory
// at head_dim 128, so two CTAs share an SM and one CTA's softmax runs under the other's
// MMAs. tcgen05.commit on an mbarrier marks
// the end of each tile's S (and of every earlier MMA: they complete in order). V rows past
// the context in the last tile are zeroed before P V (an unused slot may hold NaN, and
// 0 * NaN is NaN). Warp-collective tcgen05 loads and stores always run on a path every
// thread of the warp takes. Every wait is bounded: a timeout sets PI_ERR_TIMEOUT, the CTA
// drains its loads and MMAs, frees its TMEM and exits.
#include <cudaTypedefs.h>

#include <type_traits>

#include "pi_common.cuh"
#include "umma_desc.cuh"

namespace pi {
namespace attn {
// Cached 2-D tensor map over a physical pool [rows = P*Hkv*S, D] (paged_decode_attn.cu).
bool pool_tensor_map(CUtensorMap* out, const void* base, uint64_t rows, int D, int S, int dtype);
}  // namespace attn

namespace prefill_tc {
namespace {

constexpr int kThreads = 128;
constexpr int kM = 128;       // query rows per CTA = TMEM lanes
constexpr int kN = 64;        // keys per tile
constexpr int kKSlots = 2;    // K ring
constexpr int kVSlots = 2;    // V ring
constexpr uint32_t kOCol = 64;  // S in TMEM columns [0, 64), O in [64, 64 + D)
constexpr float kRescaleLog2 = 8.0f;  // a row's running maximum moves by more than this only

template <int D, int S>
struct Cfg {
  static constexpr int kBoxes = D / 64;                   // 64-element (128-byte) column boxes
  static constexpr int kQBoxBytes = kM * 128;
  static constexpr int kKVBoxBytes = kN * 128;
  static constexpr int kQBytes = kBoxes * kQBoxBytes;     // Q tile [boxes][128 rows][128 B]
  static constexpr int kKVBytes = kBoxes * kKVBoxBytes;   // K or V tile [boxes][64 keys][128 B]
  static constexpr int kPBytes = kM * 128;                // P [128 rows][64 keys] bf16: one box
  static constexpr int kPagesPerTile = kN / S;
  static constexpr uint32_t kTmemCols = kOCol + D <= 128 ? 128 : 256;
  static constexpr int kBarBytes = 64;                    // 5 mbarriers + TMEM address
  static constexpr int kLayoutBytes = kQBytes + (kKSlots + kVSlots) * kKVBytes + kPBytes + kBarBytes;
  // Slack for aligning the tiles to 1024 bytes (the 128-byte swizzle's period). 896 bytes
  // covers any base aligned to 128 bytes and keeps two head_dim-128 CTAs on one SM (228 KB,
  // 1 KB reserved per CTA); the kernel checks the fit and reports PI_ERR_MISALIGNED if not.
  static constexpr int kSlack = 896;
  static constexpr int kSmem = kSlack + kLayoutBytes;
};

struct Params {
  void* out;
  const void* q;
  const int32_t* block_table;
  int64_t num_pages;
  int64_t q_tok_stride;
  int64_t out_tok_stride;
  int q_len, kv_len, q_start, causal;
  int hkv, group, tokens_per_cta;
  float scale_log2;
  int* err;
};

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem], kind::f16 with an f32 accumulator; `acc` 0 overwrites.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// 32 consecutive TMEM columns of this thread's lane (32x32b shape, warp-collective).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Byte offset of 16-byte chunk `ch` (along the row) of row `r` in a [boxes][128][128 B]
// tile with the 128-byte swizzle (the layout TMA writes and the K-major descriptors read).
__device__ __forceinline__ uint32_t sw128_off(int r, int ch) {
  return static_cast<uint32_t>((ch >> 3) * (128 * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
}

template <typename T, int D, int S>
__global__ void __launch_bounds__(kThreads, 2)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap_k,
                            const __grid_constant__ CUtensorMap tmap_v, const Params p) {
  using C = Cfg<D, S>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* qs = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  uint8_t* ks = qs + C::kQBytes;                    // K slot s at s * kKVBytes
  uint8_t* vs = ks + kKSlots * C::kKVBytes;         // V slot s at s * kKVBytes
  uint8_t* ps = vs + kVSlots * C::kKVBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ps + C::kPBytes);  // K[0..1], V[0..1], MMA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kKSlots + kVSlots + 1);
  if ((qs - smem_raw) + C::kLayoutBytes > C::kSmem) {  // CTA-uniform: the base is too unaligned
    if (threadIdx.x == 0) record_error(p.err, PI_ERR_MISALIGNED);
    return;
  }

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int G = p.group;
  const int h = blockIdx.y;
  // causal: the latest (heaviest) query blocks first
  const int qblk = p.causal ? static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x)
                            : static_cast<int>(blockIdx.x);
  const int t0 = qblk * p.tokens_per_cta;
  const int t_end = min(p.q_len, t0 + p.tokens_per_cta);
  // keys any row of this CTA may see
  const int kv_hi = p.causal ? min(p.kv_len, p.q_start + t_end) : p.kv_len;
  const int n_tiles = kv_hi > 0 ? (kv_hi + kN - 1) / kN : 0;
  const int n_pages = (kv_hi + S - 1) / S;
  const uint32_t mma_bar = smem_u32(bars + kKSlots + kVSlots);

  pdl_trigger();
  pdl_wait();

  if (tid == 0) {
    for (int b = 0; b < kKSlots + kVSlots + 1; ++b) mbar_init(smem_u32(bars + b), 1);
    fence_mbar_init();
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // Q rows into the swizzled K-major tile; rows past q_len are zero
  for (int c = tid; c < kM * (D / 8); c += kThreads) {
    const int r = c / (D / 8);
    const int ch = c - r * (D / 8);
    const int tok = t0 + r / G;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (tok < p.q_len)
      v = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) +
                                          static_cast<int64_t>(tok) * p.q_tok_stride +
                                          static_cast<int64_t>(h * G + r % G) * D + ch * 8);
    *reinterpret_cast<uint4*>(qs + sw128_off(r, ch)) = v;
  }
  fence_proxy_async_smem();  // the MMA reads Q through the async proxy
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_row = tmem + (static_cast<uint32_t>(32 * warp) << 16);  // this warp's lanes

  // Page ids of tile j (thread 0). They are fetched one iteration before the loads that use
  // them, so the TMA issue never waits on a block-table read.
  auto fetch_ids = [&](int j, int (&ids)[C::kPagesPerTile]) {
#pragma unroll
    for (int pp = 0; pp < C::kPagesPerTile; ++pp) {
      const int pg = j * C::kPagesPerTile + pp;
      ids[pp] = (j < n_tiles && pg < n_pages) ? p.block_table[pg] : 0;
    }
  };
  // K (kind 0) or V (kind 1) of tile j into `dst`, completing on `bar` (thread 0).
  auto issue_load = [&](int j, int kind, uint32_t dst, uint32_t bar, const int (&ids)[C::kPagesPerTile]) {
    const int pg0 = j * C::kPagesPerTile;
    const int np = min(C::kPagesPerTile, n_pages - pg0);
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(np * C::kBoxes * S * 128));
#pragma unroll
    for (int pp = 0; pp < C::kPagesPerTile; ++pp) {
      if (pp >= np) break;
      int pid = ids[pp];
      if (pid < 0 || static_cast<int64_t>(pid) >= p.num_pages) {
        record_error(p.err, PI_ERR_PAGE_RANGE);
        pid = 0;
      }
      const int row = (pid * p.hkv + h) * S;
#pragma unroll
      for (int b = 0; b < C::kBoxes; ++b)
        tma_load_2d(dst + b * C::kKVBoxBytes + pp * S * 128, kind ? &tmap_v : &tmap_k, bar, 64 * b,
                    row);
    }
  };
  const uint32_t k_addr0 = smem_u32(ks);
  const uint32_t v_addr0 = smem_u32(vs);
  int k_issued = 0, v_issued = 0;  // loads thread 0 has issued
  // Thread 0's page ids: at the top of iteration j, ids_k holds tile j + 1's (for V(j + 1))
  // and ids_n tile j + 2's (for K(j + 2)); ids_v serves the first tile's loads.
  int ids_v[C::kPagesPerTile], ids_k[C::kPagesPerTile], ids_n[C::kPagesPerTile];
  if (tid == 0) {
    fetch_ids(0, ids_v);
    fetch_ids(1, ids_k);
    if (n_tiles > 0) issue_load(0, 0, k_addr0, smem_u32(bars + 0), ids_v);
    if (n_tiles > 0) issue_load(0, 1, v_addr0, smem_u32(bars + kKSlots), ids_v);
    if (n_tiles > 1) issue_load(1, 0, k_addr0 + C::kKVBytes, smem_u32(bars + 1), ids_k);
    if (n_tiles > 1) issue_load(1, 1, v_addr0 + C::kKVBytes, smem_u32(bars + kKSlots + 1), ids_k);
    k_issued = v_issued = min(2, n_tiles);
    fetch_ids(2, ids_n);
  }

  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const uint32_t id_s = umma::instr_desc_f16(kBf16, kM, kN, false, false);
  const uint32_t id_o = umma::instr_desc_f16(kBf16, kM, D, false, true);
  const uint32_t q_addr = smem_u32(qs);
  const uint32_t p_addr = smem_u32(ps);

  const int r = tid;  // this thread's query row and TMEM lane
  const int tok = t0 + r / G;
  const int lim = p.causal ? min(p.kv_len, p.q_start + tok + 1) : p.kv_len;
  float m_run = -INFINITY;
  float l_run = 0.f;
  uint32_t mma_phase = 0;
  int k_done = 0, v_done = 0;  // loads whose completion thread 0 has seen (for the drain)
  bool failed = false;

  for (int j = 0; j < n_tiles; ++j) {
    const int ksl = j % kKSlots;
    // ---- S = Q K^T into TMEM columns [0, 64), issued once K(j) has landed. Only thread 0
    // waits for the load; it commits even after a timeout (so the others' wait below ends)
    // and its failure reaches every thread at the barrier after that wait.
    if (tid == 0) {
      if (!failed &&
          mbar_wait_bounded(smem_u32(bars + ksl), static_cast<uint32_t>((j / kKSlots) & 1))) {
        k_done = j + 1;
        tc_fence_after();
        const uint32_t k_addr = k_addr0 + ksl * C::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t col = static_cast<uint32_t>((kk & 3) * 32);
          umma_f16(tmem,
                   umma::smem_desc(q_addr + (kk >> 2) * C::kQBoxBytes + col, 16, 1024, umma::kSwizzle128),
                   umma::smem_desc(k_addr + (kk >> 2) * C::kKVBoxBytes + col, 16, 1024, umma::kSwizzle128),
                   id_s, kk > 0 ? 1u : 0u);
        }
      } else {
        failed = true;
      }
      umma_commit(mma_bar);
    }
    if (!mbar_wait_bounded(mma_bar, mma_phase)) failed = true;
    mma_phase ^= 1u;
    if (__syncthreads_or(failed)) {
      failed = true;
      break;
    }
    tc_fence_after();
    // S(j) is done, and with it every earlier MMA (P V of tile j - 1): K slot j % 2 and V
    // slot (j + 1) % 2 are free, so K(j + 2) and V(j + 1) go out now.
    if (tid == 0) {
      if (k_issued < n_tiles && k_issued == j + kKSlots) {
        issue_load(k_issued, 0, k_addr0 + ksl * C::kKVBytes, smem_u32(bars + ksl), ids_n);
        ++k_issued;
      }
      if (j >= 1 && v_issued < n_tiles && v_issued == j + 1) {
        const int vsl = v_issued % kVSlots;
        issue_load(v_issued, 1, v_addr0 + vsl * C::kKVBytes, smem_u32(bars + kKSlots + vsl), ids_k);
        ++v_issued;
      }
      // ids_k held tile j + 1's ids, ids_n tile j + 2's; move on by one tile
#pragma unroll
      for (int pp = 0; pp < C::kPagesPerTile; ++pp) ids_k[pp] = ids_n[pp];
      fetch_ids(j + 3, ids_n);
    }
    __syncwarp();  // warp 0 converged again after thread 0's issue: the loads are .aligned
    // ---- online softmax of this row
    float sv[kN];
    tmem_ld32(t_row, sv);
    tmem_ld32(t_row + 32, sv + 32);
    tmem_wait_ld();
    const int key0 = j * kN;
    // Tiles whose keys this row sees in full (all but the causal diagonal and the last
    // tile) skip the per-key mask: the raw maximum is scaled once and each P is one FMA
    // and one exp2. Others mask by select and scale every score.
    const bool fast = key0 + kN <= lim && p.scale_log2 > 0.f;
    float mt = -INFINITY;
    if (fast) {
#pragma unroll
      for (int c = 0; c < kN; ++c) mt = fmaxf(mt, sv[c]);
      mt *= p.scale_log2;
    } else {
#pragma unroll
      for (int c = 0; c < kN; ++c) {
        sv[c] = key0 + c < lim ? sv[c] * p.scale_log2 : -INFINITY;
        mt = fmaxf(mt, sv[c]);
      }
    }
    // The running maximum moves only past a margin: P = 2^(s - m) stays <= 2^kRescaleLog2,
    // and O needs rescaling only on the tiles where a row's maximum jumps.
    float m_new = m_run;
    bool rescale = false;
    if (mt > m_run + kRescaleLog2) {
      rescale = m_run != -INFINITY;  // before any key O is zero: nothing to rescale
      m_new = mt;
    }
    const float alpha = rescale ? fast_exp2(m_run - m_new) : 1.f;
    float ls = 0.f;
    auto store_p = [&](int ch, const float (&pv)[8]) {
      const uint4 packed = make_uint4(MmaOp<T>::pack(pv[0], pv[1]), MmaOp<T>::pack(pv[2], pv[3]),
                                      MmaOp<T>::pack(pv[4], pv[5]), MmaOp<T>::pack(pv[6], pv[7]));
      *reinterpret_cast<uint4*>(ps + sw128_off(r, ch)) = packed;
    };
    if (fast) {
      const float neg_m = -m_new;  // finite: 64 visible keys
#pragma unroll
      for (int ch = 0; ch < kN / 8; ++ch) {
        float pv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          pv[e] = fast_exp2(fmaf(sv[ch * 8 + e], p.scale_log2, neg_m));
          ls += pv[e];
        }
        store_p(ch, pv);
      }
    } else {
#pragma unroll
      for (int ch = 0; ch < kN / 8; ++ch) {
        float pv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float x = sv[ch * 8 + e];
          pv[e] = x == -INFINITY ? 0.f : fast_exp2(x - m_new);
          ls += pv[e];
        }
        store_p(ch, pv);
      }
    }
    l_run = l_run * alpha + ls;
    m_run = m_new;
    // ---- O of earlier tiles, rescaled where a row's maximum moved (P V of tile j - 1 is
    // complete). The TMEM loads are warp-collective: the whole warp takes the branch.
    if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float ov[32];
        tmem_ld32(t_row + kOCol + 32 * c, ov);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) ov[e] *= alpha;
        tmem_st32(t_row + kOCol + 32 * c, ov);
      }
      tmem_wait_st();
    }
    // ---- V(j): on the last tile every thread waits for it and zeroes the rows past the
    // context (they may hold NaN); otherwise only the MMA issuer waits, below.
    const int vsl = j % kVSlots;
    const uint32_t v_bar = smem_u32(bars + kKSlots + vsl);
    const uint32_t v_parity = static_cast<uint32_t>((j / kVSlots) & 1);
    const int valid = min(kN, kv_hi - key0);
    if (valid < kN) {
      if (!mbar_wait_bounded(v_bar, v_parity)) failed = true;
      if (__syncthreads_or(failed)) {
        failed = true;
        break;
      }
      if (tid == 0) v_done = j + 1;
      uint8_t* vs_j = vs + vsl * C::kKVBytes;
      const int per_box = (kN - valid) * 8;
      for (int c = tid; c < C::kBoxes * per_box; c += kThreads) {
        const int b = c / per_box;
        const int rem = c - b * per_box;
        *reinterpret_cast<uint4*>(vs_j + b * C::kKVBoxBytes + (valid + rem / 8) * 128 + (rem & 7) * 16) =
            make_uint4(0u, 0u, 0u, 0u);
      }
    }
    fence_proxy_async_smem();  // P and the zeroed V rows are read by the MMA
    tc_fence_before();
    __syncthreads();
    // ---- O += P V into TMEM columns [64, 64 + D)
    if (tid == 0) {
      if (valid == kN && !failed) {
        if (mbar_wait_bounded(v_bar, v_parity))
          v_done = j + 1;
        else
          failed = true;
      }
      if (!failed) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kN / 16; ++kk) {
          const uint64_t a = umma::smem_desc(p_addr + static_cast<uint32_t>(kk * 32), 16, 1024,
                                             umma::kSwizzle128);
          const uint64_t b = umma::smem_desc(v_addr0 + static_cast<uint32_t>(vsl * C::kKVBytes + kk * 16 * 128),
                                             C::kKVBoxBytes, 1024, umma::kSwizzle128);
          umma_f16(tmem + kOCol, a, b, id_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
      }
    }
  }

  // ---- wait for the last P V (and, after a failure, for whatever MMA was issued)
  if (n_tiles > 0) {
    if (tid == 0) umma_commit(mma_bar);
    if (!mbar_wait_bounded(mma_bar, mma_phase)) failed = true;
  }
  failed = __syncthreads_or(failed) != 0;
  tc_fence_after();
  if (failed) {
    if (tid == 0) {
      record_error(p.err, PI_ERR_TIMEOUT);
      // loads still in flight must land before the CTA's shared memory is released
      for (int j = k_done; j < k_issued; ++j)
        mbar_wait_bounded(smem_u32(bars + (j % kKSlots)), static_cast<uint32_t>((j / kKSlots) & 1));
      for (int j = v_done; j < v_issued; ++j)
        mbar_wait_bounded(smem_u32(bars + kKSlots + (j % kVSlots)),
                          static_cast<uint32_t>((j / kVSlots) & 1));
    }
  } else {
    // The TMEM loads are warp-collective (.sync.aligned): every thread of the CTA runs
    // them on the same path, rows past q_len included (a warp can straddle q_len); only
    // the stores depend on the row.
    const bool row_valid = tok < p.q_len;
    T* orow = static_cast<T*>(p.out) +
              static_cast<int64_t>(row_valid ? tok : 0) * p.out_tok_stride +
              static_cast<int64_t>(h * G + r % G) * D;
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      float ov[32];
      if (n_tiles > 0) {
        tmem_ld32(t_row + kOCol + 32 * c, ov);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) ov[e] = 0.f;
      }
      if (row_valid) {
#pragma unroll
        for (int e = 0; e < 32; e += 2)
          *reinterpret_cast<uint32_t*>(orow + 32 * c + e) =
              MmaOp<T>::pack(ov[e] * inv, ov[e + 1] * inv);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(C::kTmemCols)
                 : "memory");
  }
}

bool configured[64][8] = {};

template <typename T, int D, int S>
int launch(const Params& p, int n_qblocks, const CUtensorMap& tk, const CUtensorMap& tv,
           cudaStream_t stream) {
  using C = Cfg<D, S>;
  auto kern = paged_prefill_tc_kernel<T, D, S>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return PI_ERR_CUDA;
  const int slot = (std::is_same<T, __half>::value ? 4 : 0) + (D == 128 ? 2 : 0) + (S == 32 ? 1 : 0);
  if (!configured[dev][slot]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) != cudaSuccess)
      return PI_ERR_CUDA;
    configured[dev][slot] = true;
  }
  const cudaError_t e =
      launch_kernel(kern, dim3(n_qblocks, p.hkv), dim3(kThreads), C::kSmem, stream, tk, tv, p);
  return e == cudaSuccess ? PI_OK : PI_ERR_CUDA;
}

}  // namespace
}  // namespace prefill_tc
}  // namespace pi

extern "C" int pi_paged_prefill_attn_tc(void* out, const void* q, const void* k_pool,
                                        const void* v_pool, const int32_t* block_table,
                                        int64_t table_len, int q_len, int kv_len, int q_start,
                                        int causal, int num_q_heads, int num_kv_heads,
                                        int head_dim, int page_size, int64_t num_pages,
                                        float scale, int dtype, int64_t q_tok_stride,
                                        int64_t out_tok_stride, int* err, cudaStream_t stream) {
  using namespace pi;
  if (dtype != PI_DTYPE_BF16 && dtype != PI_DTYPE_F16) return PI_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return PI_ERR_UNSUPPORTED;
  if (page_size != 16 && page_size != 32) return PI_ERR_UNSUPPORTED;
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads) return PI_ERR_BAD_SHAPE;
  const int G = num_q_heads / num_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8 && G != 16) return PI_ERR_UNSUPPORTED;
  if (q_len < 0 || kv_len < 0 || q_start < 0 || num_pages <= 0 || table_len < 0) return PI_ERR_BAD_SHAPE;
  if (static_cast<int64_t>(kv_len) > table_len * page_size) return PI_ERR_BAD_SHAPE;
  if (q_tok_stride < static_cast<int64_t>(num_q_heads) * head_dim ||
      out_tok_stride < static_cast<int64_t>(num_q_heads) * head_dim)
    return PI_ERR_BAD_SHAPE;
  if (static_cast<int64_t>(num_pages) * num_kv_heads * page_size > (int64_t{1} << 31))
    return PI_ERR_BAD_SHAPE;  // TMA row coordinate is a 32-bit int
  if (q_len == 0) return PI_OK;
  if (!out || !q || !k_pool || !v_pool || (kv_len > 0 && !block_table)) return PI_ERR_NULL_POINTER;
  // Q rows are read as 16-byte vectors, outputs written as element pairs
  if (!aligned(q, 16) || (q_tok_stride % 8) || !aligned(out, 4) || (out_tok_stride % 2) ||
      !aligned(k_pool, 16) || !aligned(v_pool, 16))
    return PI_ERR_MISALIGNED;
  const uint64_t rows = static_cast<uint64_t>(num_pages) * num_kv_heads * page_size;
  CUtensorMap tk, tv;
  if (!attn::pool_tensor_map(&tk, k_pool, rows, head_dim, page_size, dtype) ||
      !attn::pool_tensor_map(&tv, v_pool, rows, head_dim, page_size, dtype))
    return PI_ERR_CUDA;
  prefill_tc::Params p;
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
  p.tokens_per_cta = 128 / G;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = err;
  const int n_qblocks = (q_len + p.tokens_per_cta - 1) / p.tokens_per_cta;
#define PI_PREFILL_TC(T, D, S)                                  \
  if (head_dim == D && page_size == S)                          \
    return prefill_tc::launch<T, D, S>(p, n_qblocks, tk, tv, stream);
  if (dtype == PI_DTYPE_BF16) {
    PI_PREFILL_TC(__nv_bfloat16, 64, 16)
    PI_PREFILL_TC(__nv_bfloat16, 128, 16)
    PI_PREFILL_TC(__nv_bfloat16, 64, 32)
    PI_PREFILL_TC(__nv_bfloat16, 128, 32)
  } else {
    PI_PREFILL_TC(__half, 64, 16)
    PI_PREFILL_TC(__half, 128, 16)
    PI_PREFILL_TC(__half, 64, 32)
    PI_PREFILL_TC(__half, 128, 32)
  }
#undef PI_PREFILL_TC
  return PI_ERR_UNSUPPORTED;
}
