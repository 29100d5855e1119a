// Paged prefill attention on the 5th-generation tensor cores (tcgen05, TMEM accumulators).
//
// Same operation and arguments as pi_paged_prefill_attn (paged_prefill_attn.cu), which
// replaces the prefill branch of the reference's _attn_paged
// (src/plastic_infer/exec/runner_paged.py:36-95):
//   out[i, hq] = softmax(scale * q[i, hq] . K[hq / G]^T) V[hq / G]  over keys j < lim(i),
//   lim(i) = min(kv_len, q_start + i + 1) when causal, kv_len otherwise.
//
// CTA = (block of 128 / G query tokens, KV head): 128 query rows, row r = token * G + g,
// one row per TMEM lane. The context streams in tiles of 64 keys (64 / S pages by TMA).
// Warp-specialized, six warps, synchronized only through mbarriers (full / empty pairs):
//   - load warp: TMA of the Q tile (a 3-D box of G heads x 128 / G tokens per 64 columns,
//     zero past q_len), then K(t) and V(t) into 2-slot rings, each slot reloaded once the
//     MMA that read it has completed;
//   - MMA warp (one thread): S(t) = Q K(t)^T into one of two TMEM buffers (columns [0, 64)
//     and [64, 128)) as soon as K(t) has landed and the softmax has read that buffer's
//     previous S, then O += P(t - 1) V(t - 1) (columns [128, 128 + D)) with P read from
//     TMEM as the A operand; kind::f16, M = 128, K-major Q and K with the 128-byte swizzle,
//     MN-major V;
//   - 4 softmax warps (one thread per row): read S(t), release its buffer, run the online
//     softmax in base 2, write P (bf16/f16 pairs) over the first 32 columns of S(t)'s
//     buffer, rescale O where needed (after the previous P V), then signal P ready.
// P(t) overwrites S(t) in place: the MMA thread issues S(t + 2) into that buffer only after
// P(t) V(t), and one thread's tcgen05.mma run in order.
// So S(t + 1) computes while the softmax of tile t runs, and the softmax never waits on a
// load. The running maximum of a row moves only when it grows by more than 2^8: P <= 256,
// and O is rescaled on those rare tiles only (the stale maximum cancels in O / l). Tiles a
// row sees in full skip the per-key mask (one FMA and one exp2 per score). V rows past the
// context in the last tile are zeroed before P V (an unused slot may hold NaN, and
// 0 * NaN is NaN). At the end each softmax warp writes its 32 rows of O / l into the Q
// tile's space and stores them with one TMA store per 64 columns (rows of tokens past q_len
// are dropped by the store). Warp-collective tcgen05 loads and stores run on a path every
// thread of the warp takes. The CTA needs 97 KB of shared memory and 256 TMEM columns at
// head_dim 128, so two CTAs share an SM. Every wait is bounded: a timeout sets
// PI_ERR_TIMEOUT, the roles leave their loops, in-flight loads and MMAs complete, TMEM is
// freed.
#include <cudaTypedefs.h>

#include <type_traits>

#include "pi_common.cuh"
#include "umma_desc.cuh"

namespace pi {
namespace attn {
// Cached 2-D tensor map over a physical pool [rows = P*Hkv*S, D], and the driver's tensor-map
// encoder (paged_decode_attn.cu).
bool pool_tensor_map(CUtensorMap* out, const void* base, uint64_t rows, int D, int S, int dtype);
PFN_cuTensorMapEncodeTiled_v12000 get_encode();
}  // namespace attn

namespace prefill_tc {
namespace {

constexpr int kSoftmaxWarps = 4;  // one per TMEM lane quadrant, one thread per query row
constexpr int kMmaWarp = 4;       // issues every tcgen05.mma (lane 0)
constexpr int kLoadWarp = 5;      // issues every TMA load (lane 0)
constexpr int kThreads = 32 * 6;
constexpr int kM = 128;       // query rows per CTA = TMEM lanes
constexpr int kN = 64;        // keys per tile
constexpr int kKSlots = 2;    // K ring
constexpr int kVSlots = 2;    // V ring
constexpr uint32_t kOCol = 128;  // S double-buffered in TMEM columns [0, 64) and [64, 128),
                                 // O in [128, 128 + D)
constexpr uint32_t kTmemCols = 256;
constexpr float kRescaleLog2 = 8.0f;  // a row's running maximum moves by more than this only

template <int D, int S>
struct Cfg {
  static constexpr int kBoxes = D / 64;                   // 64-element (128-byte) column boxes
  static constexpr int kQBoxBytes = kM * 128;
  static constexpr int kKVBoxBytes = kN * 128;
  static constexpr int kQBytes = kBoxes * kQBoxBytes;     // Q tile [boxes][128 rows][128 B]
  static constexpr int kKVBytes = kBoxes * kKVBoxBytes;   // K or V tile [boxes][64 keys][128 B]
  static constexpr int kPagesPerTile = kN / S;
  static constexpr int kBarBytes = 144;  // 17 mbarriers + TMEM address
  static constexpr int kLayoutBytes = kQBytes + (kKSlots + kVSlots) * kKVBytes + kBarBytes;
  // Slack for aligning the tiles to 1024 bytes (the 128-byte swizzle's period). 768 bytes
  // covers any base aligned to 256 bytes and keeps two head_dim-128 CTAs on one SM (228 KB,
  // 1 KB reserved per CTA); the kernel checks the fit and reports PI_ERR_MISALIGNED if not.
  static constexpr int kSlack = 768;
  static constexpr int kSmem = kSlack + kLayoutBytes;
  // Dynamic shared memory requested at launch: at least 80 KB, so that at most two CTAs
  // share an SM and their 2 x 256 TMEM columns fit its 512 (tcgen05.alloc never waits).
  static constexpr int kLaunchSmem = kSmem > 80 * 1024 ? kSmem : 80 * 1024;
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

// Paired fp32 arithmetic of sm_100 (fma / add on two lanes of a 64-bit register pair): each
// lane is the IEEE round-to-nearest result of its scalar operation.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// D[tmem] (+)= A[tmem] * B[smem], kind::f16 with an f32 accumulator.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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

// 3-D tiled TMA load global -> shared (coordinates innermost first), completion on `bar`.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, uint32_t bar, int x,
                                            int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(tmap), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 3-D tiled TMA store shared -> global; elements outside the tensor are not written.
__device__ __forceinline__ void tma_store_3d(const void* tmap, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];"
               ::"l"(tmap), "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}

// Commit this thread's bulk stores and wait until their shared-memory sources have been read.
__device__ __forceinline__ void tma_store_commit_wait_read() {
  asm volatile("cp.async.bulk.commit_group;\n\tcp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Barrier slots (mbarriers in shared memory): full / empty pairs of the K and V rings and
// of the two S buffers, P ready, P V done, a one-phase drain barrier and Q landed.
enum Bar : int {
  kKFull = 0,    // [2] K(t) landed (TMA bytes)
  kKEmpty = 2,   // [2] S(t) complete: K slot free (MMA commit)
  kVFull = 4,    // [2] V(t) landed
  kVEmpty = 6,   // [2] P V(t) complete: V slot free
  kSFull = 8,    // [2] S(t) complete (MMA commit)
  kSEmpty = 10,  // [2] S(t) read by the 4 softmax warps
  kPFull = 12,   // [2] P(t) in TMEM and O rescaled (4 softmax warps), slot t % 2: a warp
                 // may run a tile ahead of another (it waits for the previous P V only to
                 // rescale), and tile t + 1's arrivals must not complete tile t's phase
  kOFree = 14,   // P V(t) complete: O free (MMA commit)
  kDrain = 15,   // every MMA issued has completed (one phase, at the end)
  kQFull = 16,   // the Q tile landed (TMA bytes, one phase)
  kNumBars = 17,
};
static_assert(kNumBars * 8 + 4 <= 144, "the mbarriers and the TMEM address fit kBarBytes");

template <typename T, int D, int S>
__global__ void __launch_bounds__(kThreads, 2)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap_k,
                            const __grid_constant__ CUtensorMap tmap_v,
                            const __grid_constant__ CUtensorMap tmap_q,
                            const __grid_constant__ CUtensorMap tmap_o, const Params p) {
  using C = Cfg<D, S>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* qs = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  uint8_t* ks = qs + C::kQBytes;                    // K slot s at s * kKVBytes
  uint8_t* vs = ks + kKSlots * C::kKVBytes;         // V slot s at s * kKVBytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(vs + kVSlots * C::kKVBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  if ((qs - smem_raw) + C::kLayoutBytes > C::kSmem) {  // CTA-uniform: the base is too unaligned
    if (threadIdx.x == 0) record_error(p.err, PI_ERR_MISALIGNED);
    return;
  }
  auto bar = [&](int i) { return smem_u32(bars + i); };

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = p.group;
  // One CTA per (query block, KV head), KV head fastest. CTAs start in index order, so with
  // causal masking the latest (heaviest) query blocks of every head go first and the light
  // ones fill the last wave.
  const int h = static_cast<int>(blockIdx.x) % p.hkv;
  const int n_qblocks = static_cast<int>(gridDim.x) / p.hkv;
  const int qi = static_cast<int>(blockIdx.x) / p.hkv;
  const int qblk = p.causal ? n_qblocks - 1 - qi : qi;
  const int t0 = qblk * p.tokens_per_cta;
  const int t_end = min(p.q_len, t0 + p.tokens_per_cta);
  // keys any row of this CTA may see
  const int kv_hi = p.causal ? min(p.kv_len, p.q_start + t_end) : p.kv_len;
  const int n_tiles = kv_hi > 0 ? (kv_hi + kN - 1) / kN : 0;
  const int n_pages = (kv_hi + S - 1) / S;

  pdl_trigger();
  pdl_wait();

  if (tid == 0) {
    for (int b = 0; b < kNumBars; ++b)
      mbar_init(bar(b), (b == kSEmpty || b == kSEmpty + 1 || b == kPFull || b == kPFull + 1)
                            ? kSoftmaxWarps : 1);
    fence_mbar_init();
  }
  if (warp == kLoadWarp && lane == 0) {
    prefetch_tmap(&tmap_q);
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
  } else if (warp < kSoftmaxWarps && lane == 0) {
    prefetch_tmap(&tmap_o);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t k_addr0 = smem_u32(ks);
  const uint32_t v_addr0 = smem_u32(vs);
  bool failed = false;
  // Every wait is bounded. A role whose wait times out leaves its loop at once; the roles
  // waiting on it then time out too, and all meet at the barrier after the loops.

  if (warp == kLoadWarp) {
    // ---------------- TMA producer: K(t) and V(t) into slot t % 2 ----------------
    int issued[2] = {0, 0};  // K and V loads issued (tiles 0 .. issued - 1)
    if (lane == 0 && n_tiles > 0) {
      // Q rows of this CTA: box (64 columns, G heads, 128 / G tokens) per 64 columns, rows
      // r = token * G + g in the 128-byte-swizzled K-major layout; tokens past q_len are
      // filled with zeros.
      mbar_arrive_expect_tx(bar(kQFull), static_cast<uint32_t>(C::kQBytes));
#pragma unroll
      for (int b = 0; b < C::kBoxes; ++b)
        tma_load_3d(smem_u32(qs) + b * C::kQBoxBytes, &tmap_q, bar(kQFull), 64 * b, h * G, t0);
    }
    if (lane == 0) {
      for (int t = 0; t < n_tiles; ++t) {
        const int sl = t % kKSlots;
        const uint32_t free_parity = static_cast<uint32_t>(((t / kKSlots) & 1) ^ 1);
        const int pg0 = t * C::kPagesPerTile;
        const int np = min(C::kPagesPerTile, n_pages - pg0);
        int ids[C::kPagesPerTile];
#pragma unroll
        for (int pp = 0; pp < C::kPagesPerTile; ++pp) {
          int pid = pp < np ? p.block_table[pg0 + pp] : 0;
          if (pid < 0 || static_cast<int64_t>(pid) >= p.num_pages) {
            record_error(p.err, PI_ERR_PAGE_RANGE);
            pid = 0;
          }
          ids[pp] = pid;
        }
        const uint32_t bytes = static_cast<uint32_t>(np * C::kBoxes * S * 128);
        for (int kind = 0; kind < 2; ++kind) {
          if (!mbar_wait_bounded(bar((kind ? kVEmpty : kKEmpty) + sl), free_parity)) {
            failed = true;
            break;
          }
          const uint32_t full = bar((kind ? kVFull : kKFull) + sl);
          const uint32_t dst = (kind ? v_addr0 : k_addr0) + sl * C::kKVBytes;
          mbar_arrive_expect_tx(full, bytes);
#pragma unroll
          for (int pp = 0; pp < C::kPagesPerTile; ++pp) {
            if (pp >= np) break;
            const int row = (ids[pp] * p.hkv + h) * S;
#pragma unroll
            for (int b = 0; b < C::kBoxes; ++b)
              tma_load_2d(dst + b * C::kKVBoxBytes + pp * S * 128, kind ? &tmap_v : &tmap_k, full,
                          64 * b, row);
          }
          issued[kind] = t + 1;
        }
        if (failed) break;
      }
    }
    __syncwarp();
    failed = __syncthreads_or(failed) != 0;
    // after a failure, loads still in flight land before the shared memory is released
    if (failed && lane == 0) {
      if (n_tiles > 0) mbar_wait_bounded(bar(kQFull), 0);
      for (int kind = 0; kind < 2; ++kind) {
        for (int sl = 0; sl < kKSlots && sl < issued[kind]; ++sl) {
          // the last tile loaded into slot sl: its phase completes after the earlier ones
          const int last = issued[kind] - 1 - ((issued[kind] - 1 - sl) % kKSlots);
          mbar_wait_bounded(bar((kind ? kVFull : kKFull) + sl),
                            static_cast<uint32_t>((last / kKSlots) & 1));
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer: S(t) = Q K(t)^T, then P V(t - 1) ----------------
    if (lane == 0) {
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      const uint32_t id_s = umma::instr_desc_f16(kBf16, kM, kN, false, false);
      const uint32_t id_o = umma::instr_desc_f16(kBf16, kM, D, false, true);
      const uint32_t q_addr = smem_u32(qs);
      auto pv = [&](int u) {  // O += P(u) V(u)
        const int sl = u % kVSlots;
        if (!mbar_wait_bounded(bar(kPFull + u % 2), static_cast<uint32_t>((u / 2) & 1)) ||
            !mbar_wait_bounded(bar(kVFull + sl), static_cast<uint32_t>((u / kVSlots) & 1))) {
          failed = true;
          return;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kN / 16; ++kk) {
          const uint64_t b = umma::smem_desc(
              v_addr0 + static_cast<uint32_t>(sl * C::kKVBytes + kk * 16 * 128), C::kKVBoxBytes,
              1024, umma::kSwizzle128);
          umma_f16_ts(tmem + kOCol, tmem + static_cast<uint32_t>(kN * (u % 2) + 8 * kk), b, id_o,
                      (u > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(bar(kOFree));
        umma_commit(bar(kVEmpty + sl));
      };
      if (n_tiles > 0 && !mbar_wait_bounded(bar(kQFull), 0)) failed = true;
      for (int t = 0; t < n_tiles && !failed; ++t) {
        const int sl = t % kKSlots;
        const uint32_t parity = static_cast<uint32_t>((t / kKSlots) & 1);
        if (!mbar_wait_bounded(bar(kKFull + sl), parity) ||
            !mbar_wait_bounded(bar(kSEmpty + sl), parity ^ 1u)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = k_addr0 + sl * C::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t col = static_cast<uint32_t>((kk & 3) * 32);
          umma_f16(tmem + static_cast<uint32_t>(kN * sl),
                   umma::smem_desc(q_addr + (kk >> 2) * C::kQBoxBytes + col, 16, 1024, umma::kSwizzle128),
                   umma::smem_desc(k_addr + (kk >> 2) * C::kKVBoxBytes + col, 16, 1024, umma::kSwizzle128),
                   id_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(bar(kSFull + sl));
        umma_commit(bar(kKEmpty + sl));
        if (t >= 1) pv(t - 1);
      }
      if (!failed && n_tiles > 0) pv(n_tiles - 1);
      umma_commit(bar(kDrain));  // arrives once every MMA issued above has completed
    }
    __syncwarp();
    failed = __syncthreads_or(failed) != 0;
  } else {
    // ---------------- softmax warps: one thread per query row / TMEM lane ----------------
    const int r = tid;
    const uint32_t t_row = tmem + (static_cast<uint32_t>(32 * warp) << 16);  // this warp's lanes
    const int tok = t0 + r / G;
    const int lim = p.causal ? min(p.kv_len, p.q_start + tok + 1) : p.kv_len;
    float m_run = -INFINITY;
    float l_run = 0.f;
    for (int j = 0; j < n_tiles; ++j) {
      const int sb = j % 2;
      if (!mbar_wait_bounded(bar(kSFull + sb), static_cast<uint32_t>((j / 2) & 1))) failed = true;
      if (__any_sync(0xffffffffu, failed)) {
        failed = true;
        break;
      }
      tc_fence_after();
      float sv[kN];
      tmem_ld32(t_row + static_cast<uint32_t>(kN * sb), sv);
      tmem_ld32(t_row + static_cast<uint32_t>(kN * sb + 32), sv + 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kSEmpty + sb));  // S buffer sb may be overwritten
      const int key0 = j * kN;
      // Tiles whose keys this row sees in full (all but the causal diagonal and the last
      // tile) skip the per-key mask: the raw maximum is scaled once and each P is one FMA
      // and one exp2. Others mask by select and scale every score.
      const bool fast = key0 + kN <= lim && p.scale_log2 > 0.f;
      // row maximum over 8 independent chains (fmaxf is exact: the order does not matter)
      float mx[8];
      if (fast) {
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = sv[i];
#pragma unroll
        for (int c = 8; c < kN; ++c) mx[c & 7] = fmaxf(mx[c & 7], sv[c]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
#pragma unroll
        for (int c = 0; c < kN; ++c) {
          sv[c] = key0 + c < lim ? sv[c] * p.scale_log2 : -INFINITY;
          mx[c & 7] = fmaxf(mx[c & 7], sv[c]);
        }
      }
      float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                       fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      if (fast) mt *= p.scale_log2;
      // The running maximum moves only past a margin: P = 2^(s - m) stays <= 2^kRescaleLog2,
      // and O needs rescaling only on the tiles where a row's maximum jumps.
      float m_new = m_run;
      bool rescale = false;
      if (mt > m_run + kRescaleLog2) {
        rescale = m_run != -INFINITY;  // before any key O is zero: nothing to rescale
        m_new = mt;
      }
      const float alpha = rescale ? fast_exp2(m_run - m_new) : 1.f;
      uint32_t pk[kN / 2];  // P as packed pairs
      uint64_t acc[4];      // 4 independent paired partial sums of P
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = 0ull;  // +0.0f in both lanes
      if (fast) {
        const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2);
        const uint64_t neg_m2 = f2_pack(-m_new, -m_new);  // finite: 64 visible keys
#pragma unroll
        for (int c = 0; c < kN; c += 2) {
          float xa, xb;
          f2_unpack(f2_fma(f2_pack(sv[c], sv[c + 1]), scale2, neg_m2), xa, xb);
          const float a = fast_exp2(xa);
          const float b = fast_exp2(xb);
          acc[(c / 2) & 3] = f2_add(acc[(c / 2) & 3], f2_pack(a, b));
          pk[c / 2] = MmaOp<T>::pack(a, b);
        }
      } else {
#pragma unroll
        for (int c = 0; c < kN; c += 2) {
          const float a = sv[c] == -INFINITY ? 0.f : fast_exp2(sv[c] - m_new);
          const float b = sv[c + 1] == -INFINITY ? 0.f : fast_exp2(sv[c + 1] - m_new);
          acc[(c / 2) & 3] = f2_add(acc[(c / 2) & 3], f2_pack(a, b));
          pk[c / 2] = MmaOp<T>::pack(a, b);
        }
      }
      float ls_a, ls_b;
      f2_unpack(f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3])), ls_a, ls_b);
      const float ls = ls_a + ls_b;
      l_run = l_run * alpha + ls;
      m_run = m_new;
      {
        // P(t) as bf16/f16 pairs over the first 32 columns of S(t)'s buffer (read above),
        // the layout the P V MMA takes its A operand in
        float pf[kN / 2];
#pragma unroll
        for (int c = 0; c < kN / 2; ++c) pf[c] = __uint_as_float(pk[c]);
        tmem_st32(t_row + static_cast<uint32_t>(kN * sb), pf);
        tmem_wait_st();
      }
      // O of earlier tiles, rescaled where a row's maximum moved, once P V(j - 1) is done.
      // The TMEM loads are warp-collective: the whole warp takes the branch.
      if (__any_sync(0xffffffffu, rescale)) {
        if (j > 0) {
          if (!mbar_wait_bounded(bar(kOFree), static_cast<uint32_t>((j - 1) & 1))) failed = true;
          if (__any_sync(0xffffffffu, failed)) {
            failed = true;
            break;
          }
          tc_fence_after();
        }
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
      // Last tile: V rows past the context are zeroed once V has landed (they may hold
      // NaN); each softmax warp zeroes a quarter of them.
      const int valid = min(kN, kv_hi - key0);
      if (valid < kN) {
        const int vsl = j % kVSlots;
        if (!mbar_wait_bounded(bar(kVFull + vsl), static_cast<uint32_t>((j / kVSlots) & 1)))
          failed = true;
        if (__any_sync(0xffffffffu, failed)) {
          failed = true;
          break;
        }
        uint8_t* vs_j = vs + vsl * C::kKVBytes;
        const int per_box = (kN - valid) * 8;
        for (int c = tid; c < C::kBoxes * per_box; c += 32 * kSoftmaxWarps) {
          const int b = c / per_box;
          const int rem = c - b * per_box;
          *reinterpret_cast<uint4*>(vs_j + b * C::kKVBoxBytes + (valid + rem / 8) * 128 +
                                    (rem & 7) * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_smem();  // the zeroed V rows are read by the MMA
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kPFull + sb));
    }
    // The last P V, and with it every MMA, completes on the drain barrier.
    if (!failed && n_tiles > 0 && !mbar_wait_bounded(bar(kDrain), 0)) failed = true;
    failed = __syncthreads_or(failed) != 0;
    tc_fence_after();
    if (!failed) {
      // O / l goes through shared memory (the Q tile's space: every MMA that read it has
      // completed) in the Q tile's layout, and each warp stores its 32 rows with one TMA
      // store per 64 columns; rows of tokens past q_len fall outside the tensor and are not
      // written. The TMEM loads are warp-collective (.sync.aligned): every thread of the
      // warp runs them, rows past q_len included.
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
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const float* o8 = ov + 8 * q4;
          *reinterpret_cast<uint4*>(qs + sw128_off(r, 4 * c + q4)) =
              make_uint4(MmaOp<T>::pack(o8[0] * inv, o8[1] * inv), MmaOp<T>::pack(o8[2] * inv, o8[3] * inv),
                         MmaOp<T>::pack(o8[4] * inv, o8[5] * inv), MmaOp<T>::pack(o8[6] * inv, o8[7] * inv));
        }
      }
      fence_proxy_async_smem();  // the TMA store reads these rows through the async proxy
      __syncwarp();
      const int w_tok = t0 + warp * (32 / G);  // this warp's first token
      if (lane == 0 && w_tok < p.q_len) {        // a box that starts past q_len is skipped
#pragma unroll
        for (int b = 0; b < C::kBoxes; ++b)
          tma_store_3d(&tmap_o, smem_u32(qs) + b * C::kQBoxBytes + warp * 32 * 128, 64 * b, h * G,
                       w_tok);
        tma_store_commit_wait_read();
      }
    }
  }

  // After a failure every MMA still has to finish before TMEM is freed: the MMA issuer's
  // last commit (the drain barrier) covers them.
  if (failed) {
    if (tid == 0) record_error(p.err, PI_ERR_TIMEOUT);
    if (warp == kMmaWarp && lane == 0) mbar_wait_bounded(bar(kDrain), 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

bool configured[64][8] = {};

// 3-D tensor map over a [tokens][heads][D] activation with a token stride of `tok_stride`
// elements (heads contiguous): box = 64 columns x G heads x `box_tokens` tokens, the
// 128-byte swizzle (one 128-byte row per (token, head) and 64 columns). Loads outside the
// tensor read zeros, stores outside it are dropped.
bool token_tensor_map(CUtensorMap* m, const void* base, int tokens, int heads, int D,
                      int64_t tok_stride, int G, int box_tokens, int dtype) {
  auto encode = attn::get_encode();
  if (!encode) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(tokens)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(tok_stride) * 2};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(G), static_cast<cuuint32_t>(box_tokens)};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUtensorMapDataType dt =
      dtype == PI_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return encode(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, int D, int S>
int launch(const Params& p, int n_qblocks, const CUtensorMap& tk, const CUtensorMap& tv,
           const CUtensorMap& tq, const CUtensorMap& to, cudaStream_t stream) {
  using C = Cfg<D, S>;
  auto kern = paged_prefill_tc_kernel<T, D, S>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return PI_ERR_CUDA;
  const int slot = (std::is_same<T, __half>::value ? 4 : 0) + (D == 128 ? 2 : 0) + (S == 32 ? 1 : 0);
  if (!configured[dev][slot]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kLaunchSmem) !=
        cudaSuccess)
      return PI_ERR_CUDA;
    configured[dev][slot] = true;
  }
  const cudaError_t e =
      launch_kernel(kern, dim3(n_qblocks * p.hkv), dim3(kThreads), C::kLaunchSmem, stream, tk, tv,
                    tq, to, p);
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
  // Q and the output move by TMA: 16-byte aligned bases and token strides
  if (!aligned(q, 16) || (q_tok_stride % 8) || !aligned(out, 16) || (out_tok_stride % 8) ||
      !aligned(k_pool, 16) || !aligned(v_pool, 16))
    return PI_ERR_MISALIGNED;
  const uint64_t rows = static_cast<uint64_t>(num_pages) * num_kv_heads * page_size;
  CUtensorMap tk, tv, tq, to;
  if (!attn::pool_tensor_map(&tk, k_pool, rows, head_dim, page_size, dtype) ||
      !attn::pool_tensor_map(&tv, v_pool, rows, head_dim, page_size, dtype) ||
      !prefill_tc::token_tensor_map(&tq, q, q_len, num_q_heads, head_dim, q_tok_stride, G, 128 / G,
                                    dtype) ||
      !prefill_tc::token_tensor_map(&to, out, q_len, num_q_heads, head_dim, out_tok_stride, G,
                                    32 / G, dtype))
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
    return prefill_tc::launch<T, D, S>(p, n_qblocks, tk, tv, tq, to, stream);
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
