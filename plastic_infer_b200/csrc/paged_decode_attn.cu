// Batched paged GQA decode attention for B200 (sm_100a).
//
// Reference behaviour (src/plastic_infer/exec/attention.py:103-190): for one request,
// gather the block table's pages into a contiguous [T, Hkv, D] copy, repeat each KV
// head G = Hq/Hkv times, and run scaled_dot_product_attention (scale 1/sqrt(D),
// softmax over the first kv_num_tokens tokens). Query head hq reads KV head hq // G.
// The decode caller (_attn_paged, src/plastic_infer/exec/runner_paged.py:36-59) passes
// one query token and causal=False.
//
// This file computes the same thing for a whole batch in one launch, reading each KV
// byte of the pool exactly once and never materialising the gather.
//
// Fast path (bf16/f16 pools, head_dim 64/128/256, page_size 16/32, G <= 8):
//   * Work = the flattened stream of (request b, kv head h, page p) over all requests,
//     cut into equal contiguous ranges, one per resident warp (persistent grid of
//     SM-count x occupancy CTAs). Every warp reads the same number of pages, so the
//     ragged contexts cost no tail imbalance.
//   * Each warp owns a kStages-deep ring of (K tile, V tile) stages in shared memory.
//     Lane 0 fills a stage with four 2-D TMA loads (128-byte swizzled boxes of
//     [page_size rows x 64 elements]) completing on that stage's mbarrier; the warp
//     refills a stage as soon as it has consumed it, so kStages pages per warp are
//     always in flight. Page ids for the next 64 stream positions are prefetched
//     into registers one block of 32 ahead.
//   * Math per page on the tensor cores (mma.sync m16n8k16, f32 accumulate):
//       S^T[tokens, heads] = K[tokens, D] . Q^T[D, heads]   (A = K via ldmatrix)
//       O^T[D, heads]     += V^T[D, tokens] . P^T[tokens, heads]
//     The G query heads of a KV head ride in the n=8 dimension, so one K/V tile feeds
//     all of its query heads. The S^T accumulator is turned into the P^T operand with
//     movmatrix.trans; the online softmax (base-2, fp32) needs only three xor-shuffles
//     per page.
//   * A (b, h) segment cut across warps leaves fp32 partials (m, l, O) in the
//     workspace; the last warp to finish it (atomic counter) merges them and resets
//     the counter, so there is no second launch and no spin-wait anywhere.
//
// Generic path (everything else, e.g. fp32 pools or odd head_dim/page_size): one CTA
// per (request, query head), SIMT fp32, same semantics.
#include <mutex>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "pi_common.cuh"

namespace pi {
namespace attn {

// Compile-time tunables (the defaults are the measured best on B200).
#ifndef PI_ATTN_WARPS
#define PI_ATTN_WARPS 4
#endif
#ifndef PI_ATTN_MAX_STAGES
#define PI_ATTN_MAX_STAGES 4
#endif
constexpr int kWarps = PI_ATTN_WARPS;  // warps per CTA (each an independent consumer)
constexpr int kThreads = kWarps * 32;
constexpr int kMaxBatch = 4096;      // prefix table lives in shared memory
constexpr int kMaxKvHeads = 64;      // arrival counters: kMaxBatch x kMaxKvHeads
constexpr int kMaxCtasPerSm = 2;     // workspace is sized for this many
constexpr int kHeadsPad = 8;         // n dimension of the MMAs (query heads per KV head)
constexpr int64_t kL2PrefetchBytes = int64_t{48} << 20;  // pages warmed before the launch wait
constexpr unsigned kFull = 0xffffffffu;

struct FastParams {
  void* out;
  const void* q;
  const int32_t* block_tables;
  const int32_t* ctx_lens;
  int64_t bt_stride;
  int64_t q_stride;
  int64_t out_stride;
  int64_t num_pages;
  int batch;
  int hkv;
  int group;
  float scale_log2;
  int* ws_cnt;   // [batch * hkv] arrival counters (zero between launches)
  float* ws_ml;  // [n_warps * 2][kHeadsPad][2] partial (max, sum)
  float* ws_o;   // [n_warps * 2][kHeadsPad][D] partial unnormalised outputs
  int* err;
  // Fused append (all null for plain attention): before attending, request b's new
  // K/V rows k_new[b], v_new[b] ([hkv, D], row stride new_stride elements) are
  // written at slot slot_mapping[b] (< 0: none) of the pools k_pool_w / v_pool_w.
  const void* k_new;
  const void* v_new;
  const int64_t* slot_mapping;
  int64_t new_stride;
  void* k_pool_w;
  void* v_pool_w;
  // Fused peer all-gather (kGather instances only): see pi_peer_gather_t; ag_done is
  // the grid-completion counter kept in the workspace's zeroed block.
  pi_peer_gather_t ag;
  unsigned* ag_done;
};

template <int D, int S>
struct Cfg {
  static constexpr int kBoxes = D / 64;           // 128-byte column boxes per row
  static constexpr int kBoxBytes = S * 128;       // one box: S rows x 128 B
  static constexpr int kTileBytes = kBoxes * kBoxBytes;
  static constexpr int kStageBytes = 2 * kTileBytes;  // K + V
  static constexpr int kSub = S / 16;             // 16-token MMA sub-tiles per page
  static constexpr int kMT = D / 16;              // QK k-steps == PV m-tiles
};

// Pipeline depth per warp: as many (K, V) page stages as fit in ~200 KB of shared
// memory next to the batch prefix table, capped at 4 (4 x 8 KB per warp already keeps
// ~2x the bytes in flight that HBM latency needs at D = 128, 16-token pages).
template <int D, int S>
constexpr int stages_for() {
  constexpr int budget = 224 * 1024 - (kMaxBatch + 1) * 4 - 1024 - kWarps * 8 * 8;
  constexpr int n = budget / (kWarps * Cfg<D, S>::kStageBytes);
  return n < 1 ? 1 : (n > PI_ATTN_MAX_STAGES ? PI_ATTN_MAX_STAGES : n);
}

template <int D, int S, int NS>
constexpr size_t fast_smem_bytes() {
  return 1024 /* alignment slack */ + static_cast<size_t>(kWarps) * NS * Cfg<D, S>::kStageBytes +
         static_cast<size_t>(kWarps) * NS * 8 /* mbarriers */ + (kMaxBatch + 1) * 4;
}

// Byte offset of element (t, d) inside a swizzled [boxes][S][128 B] tile.
template <int S>
__device__ __forceinline__ uint32_t tile_off(int t, int d) {
  return static_cast<uint32_t>((d >> 6) * (S * 128) + t * 128 + ((((d & 63) >> 3) ^ (t & 7)) << 4));
}

__device__ __forceinline__ int clamp_pages(int ctx, int S, int64_t bt_stride) {
  const int c = ctx > 0 ? ctx : 0;
  int64_t n = (static_cast<int64_t>(c) + S - 1) / S;
  if (n > bt_stride) n = bt_stride;
  return static_cast<int>(n);
}

// Last-arriver merge of the partial results (m, l, O) of one (request, KV head)
// segment cut across `npieces` warps: out = sum_j w_j O_j / sum_j w_j l_j with
// w_j = 2^(m_j - max m). Kept out of line: it runs at most once per segment and its
// accumulators must not weigh on the page loop's register allocation.
// Where one finished row group (G query heads x D of one request) is written: this
// rank's output, and in the gather variant the same rows of every peer's gathered
// buffer (NVLink peer stores straight from registers).
template <typename T>
struct RowDsts {
  T* p[PI_MAX_PEERS];
  int n;
};

template <typename T, int D>
__device__ __noinline__ void merge_pieces(const RowDsts<T> dst, const float* ws_ml,
                                          const float* ws_o, int wa, int npieces, int role_a,
                                          int G, int lane, uint32_t stage_s, int stage_bytes) {
  // The merge sits on the launch's critical path: the segment's last piece ends with
  // the rest of the grid, and nothing else can cover its latency. So it is written
  // for latency rather than for throughput:
  // - all heads at once: lanes split into G groups of `lph` lanes, and lane (g, i)
  //   owns the float4 columns i, i + lph, i + 2 lph, ... of head g, so every read of a
  //   piece (global or shared) is contiguous across the group, and the output store of
  //   one column group is one 8-byte store;
  // - each batch's maximum first, so the pieces' weights are independent of each
  //   other (no serial exp2 chain through a running maximum);
  // - staged (stage_bytes > 0: the calling warp's page ring, idle at the end of its
  //   range): cp.async copies a batch of pieces' (O, m, l) records into shared memory
  //   at once, one L2 round trip for as many pieces as the ring holds (15 at G = 4,
  //   D = 128, 4 stages);
  // - otherwise (a merge in the middle of the range, page loads still in flight in the
  //   ring) the loads go straight to registers.
  const int gp = G <= 1 ? 1 : (G <= 2 ? 2 : (G <= 4 ? 4 : 8));
  const int lph = (32 / gp) * 4 <= D ? 32 / gp : D / 4;  // lanes per head, >= 1 float4 each
  const int g = lane / lph;
  const int li = lane % lph;
  const int n4 = D / (4 * lph);      // float4 per lane
  auto slot_of = [&](int j) { return static_cast<int64_t>(wa + j) * 2 + (j == 0 ? role_a : 0); };
  float M = -INFINITY;
  float L = 0.f;
  float4 acc[D / 16];  // n4 <= D / 16 (G = 8)
#pragma unroll
  for (int e = 0; e < D / 16; ++e) acc[e] = make_float4(0.f, 0.f, 0.f, 0.f);
  auto acc_add = [&](int e, float w, float4 v) {
    acc[e].x += w * v.x;
    acc[e].y += w * v.y;
    acc[e].z += w * v.z;
    acc[e].w += w * v.w;
  };
  // Every piece holds at least one context token, so its max is finite; the guards
  // only keep two -inf maxima (possible only with -inf scores) from making a NaN.
  auto weight = [](float m, float ref) { return m == ref ? 1.f : fast_exp2(m - ref); };
  // One piece's record in the stage: O of its G heads [G][D] fp32, then (m, l) per head.
  const int obytes = G * D * 4;
  const int rec = obytes + ((G * 8 + 15) & ~15);
  const int cap = stage_bytes / rec;
  if (cap > 0) {
    const int cpr = rec / 16;       // 16-byte chunks per record
    const int co = obytes / 16;     // ... of which O
    const uint8_t* sp = static_cast<const uint8_t*>(__cvta_shared_to_generic(stage_s));
    for (int j0 = 0; j0 < npieces; j0 += cap) {
      const int n = min(cap, npieces - j0);
      for (int q = 0; q < n; ++q) {
        const int64_t sl = slot_of(j0 + q);
        const char* os = reinterpret_cast<const char*>(ws_o + sl * kHeadsPad * D);
        const char* ms = reinterpret_cast<const char*>(ws_ml + sl * kHeadsPad * 2) - obytes;
        const uint32_t dq = stage_s + static_cast<uint32_t>(q * rec);
        for (int w = lane; w < cpr; w += 32) cp_async_16(dq + w * 16, (w < co ? os : ms) + w * 16);
      }
      cp_async_wait_all();
      __syncwarp();
      if (g < G) {
        float mb = M;
        for (int q = 0; q < n; ++q)
          mb = fmaxf(mb, *reinterpret_cast<const float*>(sp + q * rec + obytes + g * 8));
        // rescale what earlier batches accumulated
        const float a = weight(M, mb);
        M = mb;
        L *= a;
#pragma unroll
        for (int e = 0; e < D / 16; ++e) {
          acc[e].x *= a;
          acc[e].y *= a;
          acc[e].z *= a;
          acc[e].w *= a;
        }
        for (int q = 0; q < n; ++q) {
          const uint8_t* r = sp + q * rec;
          const float2 ml = *reinterpret_cast<const float2*>(r + obytes + g * 8);
          const float w = weight(ml.x, M);
          L += w * ml.y;
          const float4* v = reinterpret_cast<const float4*>(r) + g * (D / 4) + li;
#pragma unroll
          for (int e = 0; e < D / 16; ++e)
            if (e < n4) acc_add(e, w, v[e * lph]);
        }
      }
      __syncwarp();
    }
  } else if (g < G) {
#pragma unroll 8
    for (int j = 0; j < npieces; ++j) M = fmaxf(M, __ldcg(ws_ml + slot_of(j) * kHeadsPad * 2 + g * 2));
    // (at D = 256 more than one piece in flight would spill the page loop)
    constexpr int kPieceUnroll = D <= 128 ? 4 : 1;
#pragma unroll kPieceUnroll
    for (int j = 0; j < npieces; ++j) {
      const int64_t sl = slot_of(j);
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(ws_ml + sl * kHeadsPad * 2 + g * 2));
      const float w = weight(ml.x, M);
      L += w * ml.y;
      const float4* src = reinterpret_cast<const float4*>(ws_o + sl * kHeadsPad * D + g * D) + li;
#pragma unroll
      for (int e = 0; e < D / 16; ++e)
        if (e < n4) acc_add(e, w, __ldcg(src + e * lph));
    }
  }
  if (g >= G) return;
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int k = 0; k < dst.n; ++k) {
    T* row = dst.p[k] + g * D;
    const bool vec = (reinterpret_cast<uintptr_t>(row) & 7) == 0;
#pragma unroll
    for (int e = 0; e < D / 16; ++e) {
      if (e < n4) {
        T* o = row + 4 * (li + e * lph);
        const float4 x = make_float4(acc[e].x * inv, acc[e].y * inv, acc[e].z * inv, acc[e].w * inv);
        if (vec) {
          *reinterpret_cast<uint2*>(o) = make_uint2(MmaOp<T>::pack(x.x, x.y), MmaOp<T>::pack(x.z, x.w));
        } else {
          o[0] = from_f32<T>(x.x);
          o[1] = from_f32<T>(x.y);
          o[2] = from_f32<T>(x.z);
          o[3] = from_f32<T>(x.w);
        }
      }
    }
  }
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Relaxed system-scope store: callers put the fence.sys that makes it a release.
__device__ __forceinline__ void st_relaxed_sys(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <typename T, int D, int S, int NS, bool kAppend, bool kGather>
__global__ void __launch_bounds__(kThreads, 1)
    paged_decode_attn_tma_kernel(const __grid_constant__ CUtensorMap tmap_k,
                                 const __grid_constant__ CUtensorMap tmap_v, const FastParams p) {
  using C = Cfg<D, S>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* tiles = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(tiles + kWarps * NS * C::kStageBytes);
  int* s_poff = reinterpret_cast<int*>(bars + kWarps * NS);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int B = p.batch;
  const int Hkv = p.hkv;
  const int G = p.group;

  // Programmatic launch: the next kernel on the stream may launch from here on (it
  // waits for this one before it reads what this one writes).
  pdl_trigger();

  // Epoch of this gather launch: from the arguments, or one past this rank's launch
  // counter (written only by the previous launch's last warp, so every thread of this
  // launch reads the same value). Read after the programmatic wait below.
  unsigned ag_epoch = 0;
  // Exit bookkeeping of the gather variant. The last warp of the grid to finish
  // publishes `epoch` to every rank once all warps' peer stores are visible, then
  // waits until every rank has published `epoch` here: when the launch completes, the
  // whole gathered buffer is in place for whatever the stream runs next. Bounded: a
  // missing peer is reported (PI_ERR_TIMEOUT), never waited on forever.
  //
  // Ordering: each warp's peer stores precede its completion count through a GPU-scope
  // fence (release to the last warp, on the same GPU); the last warp's one system-scope
  // fence then orders everything it has observed before its flag stores (causality
  // order is transitive across the two scopes), so a rank that reads the flag with an
  // acquire load sees every row of the launch.
  auto finish = [&]() {
    if constexpr (kGather) {
      __threadfence();
      __syncwarp();
      unsigned last = 0;
      if (lane == 0) {
        const unsigned total_warps = gridDim.x * kWarps;
        last = atomicAdd(p.ag_done, 1u) == total_warps - 1;
      }
      if (last) {
        // lane 0 observed every warp's count: its fence.sys + relaxed stores release
        __threadfence_system();
        *p.ag_done = 0u;
        if (p.ag.launch_counter != nullptr) *p.ag.launch_counter = ag_epoch;
        for (int r = 0; r < p.ag.world; ++r) st_relaxed_sys(p.ag.peer_flags[r] + p.ag.rank, ag_epoch);
      }
      last = __shfl_sync(kFull, last, 0);
      if (last) {
        if (lane < p.ag.world) {
          const unsigned* f = p.ag.peer_flags[p.ag.rank] + lane;
          const uint64_t t0 = global_timer_ns();
          for (uint32_t i = 0;; ++i) {
            if (static_cast<int>(ld_acquire_sys(f) - ag_epoch) >= 0) break;
            if (i > (1u << 24) || global_timer_ns() - t0 > 2000000000ull) {
              record_error(p.err, PI_ERR_TIMEOUT);
              break;
            }
            if (i >= 4096u) __nanosleep(64);  // spin tight first: peers end within us
          }
        }
      }
    }
  };

  // Destinations of the row group at element offset `off` of this rank's output.
  auto row_dsts = [&](int64_t off) {
    RowDsts<T> d;
    d.p[0] = static_cast<T*>(p.out) + off;
    d.n = 1;
    if constexpr (kGather) {
      for (int r = 0; r < p.ag.world; ++r)
        if (r != p.ag.rank)
          d.p[d.n++] = static_cast<T*>(p.ag.peer_out[r]) +
                       static_cast<int64_t>(p.ag.rank) * p.ag.rank_stride + off;
    }
    return d;
  };

  // ---- per-CTA exclusive prefix of page counts over the batch --------------------
  {
    const int per = (B + kThreads - 1) / kThreads;
    const int beg = tid * per;
    const int end = min(beg + per, B);
    int local = 0;
    for (int i = beg; i < end; ++i) local += clamp_pages(__ldg(p.ctx_lens + i), S, p.bt_stride);
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += v;
    }
    __shared__ int warp_tot[kWarps];
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int base = 0;
    for (int w = 0; w < warp; ++w) base += warp_tot[w];
    int run = base + incl - local;
    for (int i = beg; i < end; ++i) {
      s_poff[i] = run;
      run += clamp_pages(__ldg(p.ctx_lens + i), S, p.bt_stride);
    }
    if (tid == 0) {
      int tot = 0;
      for (int w = 0; w < kWarps; ++w) tot += warp_tot[w];
      s_poff[B] = tot;
    }
  }
  const uint32_t bar0 = smem_u32(bars + warp * NS);
  if (lane == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(bar0 + 8 * s, 1);
    fence_mbar_init();
  }
  if (tid == 0) {
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
  }
  __syncthreads();

  const int NW = gridDim.x * kWarps;
  const int gw = blockIdx.x * kWarps + warp;
  const int64_t total = static_cast<int64_t>(s_poff[B]) * Hkv;
  const int hq = Hkv * G;


  // Fused append: store the step's new K/V rows in the pools (one warp per
  // (request, head) row pair). A TMA load of the same page may see the row before or
  // after this store; the warp that consumes that page patches the row in shared
  // memory from the source instead, so the result never depends on the order.
  constexpr int kRowChunks = D / 8;  // 16-byte chunks per head row
  auto append_rows = [&]() {
    if constexpr (kAppend) {
    for (int i = gw; i < B * Hkv; i += NW) {
      const int b = i / Hkv;
      const int h = i - b * Hkv;
      const int64_t s = __ldg(p.slot_mapping + b);
      if (s < 0) continue;
      if (s >= p.num_pages * S) {
        if (lane == 0) record_error(p.err, PI_ERR_SLOT_RANGE);
        continue;
      }
      const int64_t page = s / S;
      const int64_t dst = ((page * Hkv + h) * S + (s - page * S)) * D;
      const int64_t src = static_cast<int64_t>(b) * p.new_stride + static_cast<int64_t>(h) * D;
      for (int c = lane; c < 2 * kRowChunks; c += 32) {
        const bool is_v = c >= kRowChunks;
        const int cc = is_v ? c - kRowChunks : c;
        const uint4 val =
            *reinterpret_cast<const uint4*>(static_cast<const T*>(is_v ? p.v_new : p.k_new) + src + cc * 8);
        *reinterpret_cast<uint4*>(static_cast<T*>(is_v ? p.v_pool_w : p.k_pool_w) + dst + cc * 8) = val;
      }
    }
    }
  };

  // Partition over at most `total` warps so every active warp owns >= 1 page: a
  // segment's pieces are then exactly the warps [first, last] that overlap it.
  const int NWe = static_cast<int>(total < NW ? total : NW);
  const bool active = gw < NWe;
  const int64_t lo = active ? total * gw / NWe : 0;
  const int64_t hi = active ? total * (gw + 1) / NWe : 0;

  // (b, h, page) of a stream position: largest b with s_poff[b] * Hkv <= pos.
  auto locate = [&](int64_t pos, int& b, int& h, int& pg) {
    int l = 0, r = B - 1;
    while (l < r) {
      const int mid = (l + r + 1) >> 1;
      if (static_cast<int64_t>(s_poff[mid]) * Hkv <= pos) l = mid; else r = mid - 1;
    }
    b = l;
    const int n = s_poff[l + 1] - s_poff[l];
    const int64_t rem = pos - static_cast<int64_t>(s_poff[l]) * Hkv;
    h = static_cast<int>(rem / n);
    pg = static_cast<int>(rem - static_cast<int64_t>(h) * n);
  };

  // Tile index (page_id * Hkv + h) for stream position base + lane.
  auto load_ids = [&](int64_t base) -> int {
    const int64_t pos = base + lane;
    if (pos >= hi) return 0;
    int b, h, pg;
    locate(pos, b, h, pg);
    int pid = __ldg(p.block_tables + static_cast<int64_t>(b) * p.bt_stride + pg);
    if (pid < 0 || static_cast<int64_t>(pid) >= p.num_pages) {
      record_error(p.err, PI_ERR_PAGE_RANGE);
      pid = 0;
    }
    return pid * Hkv + h;
  };

  const uint32_t tiles_u32 = smem_u32(tiles) + warp * NS * C::kStageBytes;
  int64_t pbase = lo;
  int id_cur = load_ids(lo);
  int id_nxt = load_ids(lo + 32);

  // Warm L2 with this warp's first pages (lane j: page lo + j) while the previous kernel
  // on the stream may still be running. The CTAs of a programmatic launch become
  // resident as the previous grid's CTAs retire and then wait below for its tail, with
  // HBM mostly idle. A prefetch moves nothing into this CTA, and L2 is where every
  // write to device memory lands, so whatever the previous kernel still writes to these
  // pages is what the loads after the wait read. The grid prefetches at most
  // kL2PrefetchBytes, well inside L2, so the pages are still there when used.
  if (active) {
    const int64_t budget = kL2PrefetchBytes / (static_cast<int64_t>(NW) * C::kStageBytes);
    const int64_t npf = min(min(hi - lo, budget), static_cast<int64_t>(32));
    if (lane < npf) {
#pragma unroll
      for (int j = 0; j < C::kBoxes; ++j) {
        tma_prefetch_l2_2d(&tmap_k, 64 * j, id_cur * S);
        tma_prefetch_l2_2d(&tmap_v, 64 * j, id_cur * S);
      }
    }
  }

  // Everything above reads only ctx_lens and block_tables. Under a programmatic launch
  // the previous kernel on the stream may still be running up to here; from here on
  // its results (q, the pools, the launch counter) are complete and visible.
  pdl_wait();
  if constexpr (kGather) {
    ag_epoch = p.ag.launch_counter != nullptr ? __ldcg(p.ag.launch_counter) + 1u : p.ag.epoch;
  }

  // Requests with no context produce zeros (SDPA over zero keys).
  for (int b = gw; b < B; b += NW) {
    if (s_poff[b + 1] == s_poff[b]) {
      const RowDsts<T> dst = row_dsts(static_cast<int64_t>(b) * p.out_stride);
      for (int k = 0; k < dst.n; ++k)
        for (int i = lane; i < hq * D; i += 32) dst.p[k][i] = from_f32<T>(0.f);
    }
  }
  if (!active) {
    append_rows();
    finish();
    return;
  }

  auto issue = [&](int64_t pos, int stage) {
    if (pos - pbase >= 32) {
      pbase += 32;
      id_cur = id_nxt;
      id_nxt = load_ids(pbase + 32);
    }
    const int tile = __shfl_sync(kFull, id_cur, static_cast<int>(pos - pbase));
    if (lane == 0) {
      const uint32_t bar = bar0 + 8 * stage;
      const uint32_t kdst = tiles_u32 + stage * C::kStageBytes;
      const uint32_t vdst = kdst + C::kTileBytes;
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(bar, C::kStageBytes);
#pragma unroll
      for (int j = 0; j < C::kBoxes; ++j) {
        tma_load_2d(kdst + j * C::kBoxBytes, &tmap_k, bar, 64 * j, tile * S);
        tma_load_2d(vdst + j * C::kBoxBytes, &tmap_v, bar, 64 * j, tile * S);
      }
    }
  };

  int64_t issued = lo;
  for (int s = 0; s < NS && issued < hi; ++s, ++issued) issue(issued, s);
  append_rows();  // while the first pages are in flight

  // Lane-constant pieces of the fragment addressing.
  const int gid = lane >> 2;   // row group (token for S^T, d for O^T)
  const int tig = lane & 3;    // thread in group (head pair)
  const int mi = lane >> 3;    // ldmatrix matrix this lane addresses
  const int mr = lane & 7;     // row inside that matrix
  // QK: A = K[t][d], t = mr + 8*(mi&1), d = 16*kk + 8*(mi>>1)
  const int qk_t = mr + 8 * (mi & 1);
  const int qk_d = 8 * (mi >> 1);
  // PV: A = V^T, ldmatrix.trans over V[t][d], t = mr + 8*(mi>>1), d = 16*mt + 8*(mi&1)
  const int pv_t = mr + 8 * (mi >> 1);
  const int pv_d = 8 * (mi & 1);

  using Mma = MmaOp<T>;
  uint32_t qf[C::kMT][2];
  // The next segment's query fragment, loaded one segment ahead (D <= 128: at D = 256
  // the extra registers would spill the page loop, and the rows go to L2 instead).
  constexpr bool kQAhead = D <= 128;
  uint32_t qn[kQAhead ? C::kMT : 1][2];
  bool qn_valid = false;
  // Query rows of (request b, KV head h) as the MMA B fragment (heads >= G are zero).
  auto load_q = [&](int b, int h, uint32_t (*dst)[2]) {
    const T* qb = static_cast<const T*>(p.q) + static_cast<int64_t>(b) * p.q_stride +
                  static_cast<int64_t>(h) * G * D;
#pragma unroll
    for (int kk = 0; kk < C::kMT; ++kk) {
      if (gid < G) {
        const uint32_t* qr = reinterpret_cast<const uint32_t*>(qb + gid * D + 16 * kk + 2 * tig);
        dst[kk][0] = __ldg(qr);
        dst[kk][1] = __ldg(qr + 4);
      } else {
        dst[kk][0] = 0u;
        dst[kk][1] = 0u;
      }
    }
  };
  float o[C::kMT][4];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  int cb, ch, cp;
  locate(lo, cb, ch, cp);
  int cn = s_poff[cb + 1] - s_poff[cb];
  int cctx = min(max(__ldg(p.ctx_lens + cb), 0), cn * S);
  int64_t piece_start = lo;
  bool fresh = true;
  bool failed = false;
  int64_t pos = lo;
  int k = 0;
  // Fused append: the index (in the request's block table) of the page holding the
  // current segment's new slot (-1: none), the row inside it, and this lane's share
  // of the new K/V row.
  constexpr int kPatch = (2 * kRowChunks + 31) / 32;
  int patch_idx = -1;
  int patch_row = 0;
  uint4 patch_val[kPatch];

  auto first_warp_of = [&](int64_t s) -> int {
    return static_cast<int>(((s + 1) * NWe - 1) / total);
  };

  auto finalize = [&](int64_t piece_end) {
    float lt0 = l0, lt1 = l1;
#pragma unroll
    for (int x = 4; x < 32; x <<= 1) {
      lt0 += __shfl_xor_sync(kFull, lt0, x);
      lt1 += __shfl_xor_sync(kFull, lt1, x);
    }
    const int64_t seg_start = static_cast<int64_t>(s_poff[cb]) * Hkv + static_cast<int64_t>(ch) * cn;
    const int64_t seg_end = seg_start + cn;
    const int g0 = 2 * tig, g1 = 2 * tig + 1;
    if (piece_start == seg_start && piece_end == seg_end) {
      const RowDsts<T> dst = row_dsts(static_cast<int64_t>(cb) * p.out_stride +
                                      static_cast<int64_t>(ch) * G * D);
      const float i0 = lt0 > 0.f ? 1.f / lt0 : 0.f;
      const float i1 = lt1 > 0.f ? 1.f / lt1 : 0.f;
      for (int k = 0; k < dst.n; ++k) {
        T* ob = dst.p[k];
#pragma unroll
        for (int mt = 0; mt < C::kMT; ++mt) {
          const int d = 16 * mt + gid;
          if (g0 < G) {
            ob[g0 * D + d] = from_f32<T>(o[mt][0] * i0);
            ob[g0 * D + d + 8] = from_f32<T>(o[mt][2] * i0);
          }
          if (g1 < G) {
            ob[g1 * D + d] = from_f32<T>(o[mt][1] * i1);
            ob[g1 * D + d + 8] = from_f32<T>(o[mt][3] * i1);
          }
        }
      }
      return;
    }
    // Partial piece: publish (m, l, O) and let the last arriving warp merge.
    const int role = (piece_start == lo) ? 0 : 1;
    const int64_t slot = static_cast<int64_t>(gw) * 2 + role;
    float* wo = p.ws_o + slot * kHeadsPad * D;
    // only the G real heads (the MMA pads them to 8); the merge reads no others
#pragma unroll
    for (int mt = 0; mt < C::kMT; ++mt) {
      const int d = 16 * mt + gid;
      if (g0 < G) {
        wo[g0 * D + d] = o[mt][0];
        wo[g0 * D + d + 8] = o[mt][2];
      }
      if (g1 < G) {
        wo[g1 * D + d] = o[mt][1];
        wo[g1 * D + d + 8] = o[mt][3];
      }
    }
    if (gid == 0) {
      float* wml = p.ws_ml + slot * kHeadsPad * 2;
      wml[g0 * 2 + 0] = m0;
      wml[g0 * 2 + 1] = lt0;
      wml[g1 * 2 + 0] = m1;
      wml[g1 * 2 + 1] = lt1;
    }
    __threadfence();
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atomicAdd(p.ws_cnt + cb * Hkv + ch, 1);
    old = __shfl_sync(kFull, old, 0);
    const int wa = first_warp_of(seg_start);
    const int wb = static_cast<int>((seg_end * NWe - 1) / total);
    const int npieces = wb - wa + 1;
    if (old != npieces - 1) return;
    __threadfence();
    const int role_a = (total * wa / NWe == seg_start) ? 0 : 1;
    // At the end of the range every page load has been consumed: the ring is free.
    const bool ring_idle = piece_end == hi;
    merge_pieces<T, D>(row_dsts(static_cast<int64_t>(cb) * p.out_stride +
                                static_cast<int64_t>(ch) * G * D),
                       p.ws_ml, p.ws_o, wa, npieces, role_a, G, lane, tiles_u32,
                       ring_idle ? NS * C::kStageBytes : 0);
    if (lane == 0) p.ws_cnt[cb * Hkv + ch] = 0;
  };

  while (pos < hi) {
    if (fresh) {
      // New (b, h) piece: load this KV head's G query rows as the MMA B operand.
      // The fragment was loaded one segment ahead (except for the warp's first).
      if (kQAhead && qn_valid) {
#pragma unroll
        for (int kk = 0; kk < (kQAhead ? C::kMT : 1); ++kk) {
          qf[kk][0] = qn[kk][0];
          qf[kk][1] = qn[kk][1];
        }
      } else {
        load_q(cb, ch, qf);
      }
#pragma unroll
      for (int mt = 0; mt < C::kMT; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
      piece_start = pos;
      fresh = false;
      {
        // Load the next segment's query rows now, so its start does not stall on them
        // (segments follow (request, head) order, skipping empty requests, as below).
        const int64_t seg_end = static_cast<int64_t>(s_poff[cb]) * Hkv +
                                static_cast<int64_t>(ch + 1) * cn;
        qn_valid = seg_end < hi;
        if (qn_valid) {
          int nh = ch + 1, nb = cb;
          if (nh == Hkv) {
            nh = 0;
            do { ++nb; } while (nb < B && s_poff[nb + 1] == s_poff[nb]);
          }
          if constexpr (kQAhead) {
            load_q(nb, nh, qn);
          } else {
            const char* nq = reinterpret_cast<const char*>(
                static_cast<const T*>(p.q) + static_cast<int64_t>(nb) * p.q_stride +
                static_cast<int64_t>(nh) * G * D);
            if (lane * 128 < G * D * static_cast<int>(sizeof(T)))
              asm volatile("prefetch.global.L2 [%0];" ::"l"(nq + lane * 128));
          }
        }
      }
      if constexpr (kAppend) {
        // Fused append: find which of this request's pages holds its new slot and
        // fetch this head's new K/V row now (lane c holds 16-byte chunk c of
        // [K row | V row]) so the per-page check is a register compare.
        const int64_t s = __ldg(p.slot_mapping + cb);
        patch_idx = -1;
        patch_row = static_cast<int>(s % S);
        if (s >= 0 && s < p.num_pages * S) {
          const int slot_page = static_cast<int>(s / S);
          const int32_t* row = p.block_tables + static_cast<int64_t>(cb) * p.bt_stride;
          const int last = cn - 1;  // decode appends at position ctx-1: the last page
          if (__ldg(row + last) == slot_page) {
            patch_idx = last;
          } else {
            for (int j0 = 0; j0 < cn && patch_idx < 0; j0 += 32) {
              const bool hit = j0 + lane < cn && __ldg(row + j0 + lane) == slot_page;
              const unsigned m = __ballot_sync(kFull, hit);
              if (m) patch_idx = j0 + __ffs(m) - 1;
            }
          }
        }
        const int64_t src = static_cast<int64_t>(cb) * p.new_stride + static_cast<int64_t>(ch) * D;
#pragma unroll
        for (int e = 0; e < kPatch; ++e) {
          const int c = lane + 32 * e;
          if (patch_idx >= 0 && c < 2 * kRowChunks) {
            const bool is_v = c >= kRowChunks;
            const int cc = is_v ? c - kRowChunks : c;
            patch_val[e] = *reinterpret_cast<const uint4*>(
                static_cast<const T*>(is_v ? p.v_new : p.k_new) + src + cc * 8);
          }
        }
      }
    }

    const int stage = k % NS;
    if (!mbar_wait_bounded(bar0 + 8 * stage, static_cast<uint32_t>((k / NS) & 1))) {
      if (lane == 0) record_error(p.err, PI_ERR_TIMEOUT);
      failed = true;
      break;
    }
    const uint32_t ktile = tiles_u32 + stage * C::kStageBytes;
    const uint32_t vtile = ktile + C::kTileBytes;
    const int valid = min(S, cctx - cp * S);
    if (valid < S) {
      // Rows past the context may hold anything (even NaN); P is 0 there, and
      // 0 * NaN would still poison O, so clear those V rows.
      uint8_t* vt = tiles + (warp * NS + stage) * C::kStageBytes + C::kTileBytes;
      const int nrow = S - valid;
      for (int i = lane; i < C::kBoxes * nrow * 8; i += 32) {
        const int j = i / (nrow * 8);
        const int rem = i - j * nrow * 8;
        const int row = valid + rem / 8;
        const int c16 = rem & 7;
        *reinterpret_cast<uint4*>(vt + j * C::kBoxBytes + row * 128 + c16 * 16) =
            make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }
    if (kAppend && cp == patch_idx) {
      // This stage holds the page of the request's new slot: overwrite that row of
      // the K and V tiles with the new values (swizzled like the TMA box).
      uint8_t* kt = tiles + (warp * NS + stage) * C::kStageBytes;
#pragma unroll
      for (int e = 0; e < kPatch; ++e) {
        const int c = lane + 32 * e;
        if (c < 2 * kRowChunks) {
          const bool is_v = c >= kRowChunks;
          const int cc = is_v ? c - kRowChunks : c;  // chunk along D: box cc / 8, column cc % 8
          uint8_t* base = kt + (is_v ? C::kTileBytes : 0) + (cc >> 3) * C::kBoxBytes +
                          patch_row * 128 + (((cc & 7) ^ (patch_row & 7)) << 4);
          *reinterpret_cast<uint4*>(base) = patch_val[e];
        }
      }
      __syncwarp();
    }

    // S^T = K Q^T for each 16-token sub-tile.
    float s[C::kSub][4];
#pragma unroll
    for (int u = 0; u < C::kSub; ++u) {
      float ce[4] = {0.f, 0.f, 0.f, 0.f};
      float co[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < C::kMT; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(ktile + tile_off<S>(16 * u + qk_t, 16 * kk + qk_d), a0, a1, a2, a3);
        if (kk & 1) Mma::run(co, a0, a1, a2, a3, qf[kk][0], qf[kk][1]);
        else Mma::run(ce, a0, a1, a2, a3, qf[kk][0], qf[kk][1]);
      }
      const int t0 = 16 * u + gid;
      const int t1 = t0 + 8;
      s[u][0] = t0 < valid ? (ce[0] + co[0]) * p.scale_log2 : -INFINITY;
      s[u][1] = t0 < valid ? (ce[1] + co[1]) * p.scale_log2 : -INFINITY;
      s[u][2] = t1 < valid ? (ce[2] + co[2]) * p.scale_log2 : -INFINITY;
      s[u][3] = t1 < valid ? (ce[3] + co[3]) * p.scale_log2 : -INFINITY;
    }

    // Online softmax (base 2) for heads g0 = 2*tig and g1 = 2*tig + 1.
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int u = 0; u < C::kSub; ++u) {
      mx0 = fmaxf(mx0, fmaxf(s[u][0], s[u][2]));
      mx1 = fmaxf(mx1, fmaxf(s[u][1], s[u][3]));
    }
#pragma unroll
    for (int x = 4; x < 32; x <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, x));
      mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, x));
    }
    const float mn0 = fmaxf(m0, mx0);
    const float mn1 = fmaxf(m1, mx1);
    const float al0 = fast_exp2(m0 - mn0);
    const float al1 = fast_exp2(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    uint32_t pb[C::kSub][2];
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int u = 0; u < C::kSub; ++u) {
      const float p0 = fast_exp2(s[u][0] - mn0);
      const float p1 = fast_exp2(s[u][1] - mn1);
      const float p2 = fast_exp2(s[u][2] - mn0);
      const float p3 = fast_exp2(s[u][3] - mn1);
      ps0 += p0 + p2;
      ps1 += p1 + p3;
      pb[u][0] = movmatrix_trans(Mma::pack(p0, p1));
      pb[u][1] = movmatrix_trans(Mma::pack(p2, p3));
    }
    l0 = l0 * al0 + ps0;
    l1 = l1 * al1 + ps1;

    // O^T = O^T * alpha + V^T P^T.
#pragma unroll
    for (int mt = 0; mt < C::kMT; ++mt) {
      o[mt][0] *= al0;
      o[mt][1] *= al1;
      o[mt][2] *= al0;
      o[mt][3] *= al1;
#pragma unroll
      for (int u = 0; u < C::kSub; ++u) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4_trans(vtile + tile_off<S>(16 * u + pv_t, 16 * mt + pv_d), a0, a1, a2, a3);
        Mma::run(o[mt], a0, a1, a2, a3, pb[u][0], pb[u][1]);
      }
    }
    __syncwarp();

    // Refill the stage just consumed with the page NS positions ahead.
    if (issued < hi) {
      issue(issued, stage);
      ++issued;
    }
    ++k;
    ++pos;
    if (++cp == cn) {
      finalize(pos);
      if (pos < hi) {
        cp = 0;
        if (++ch == Hkv) {
          ch = 0;
          do { ++cb; } while (cb < B && s_poff[cb + 1] == s_poff[cb]);
        }
        cn = s_poff[cb + 1] - s_poff[cb];
        cctx = min(max(__ldg(p.ctx_lens + cb), 0), cn * S);
        fresh = true;
      }
    } else if (pos == hi) {
      finalize(pos);
    }
  }

  if (failed) {
    // Drain every load still in flight before the CTA's shared memory is released.
    for (int64_t j = k; j < issued - lo; ++j) {
      mbar_wait_bounded(bar0 + 8 * static_cast<int>(j % NS), static_cast<uint32_t>((j / NS) & 1));
    }
  }
  finish();
}

// ---------------------------------------------------------------------------------
// Generic SIMT path: one CTA per (request, query head); 4 warps split the pages.
// ---------------------------------------------------------------------------------

struct SimtParams {
  void* out;
  const void* q;
  const void* k_pool;
  const void* v_pool;
  const int32_t* block_tables;
  const int32_t* ctx_lens;
  int64_t bt_stride;
  int64_t q_stride;
  int64_t out_stride;
  int64_t num_pages;
  int hkv;
  int group;
  int head_dim;
  int page_size;
  float scale_log2;
  int* err;
};

constexpr int kSimtMaxD = 256;

template <typename T>
__global__ void __launch_bounds__(128) paged_decode_attn_simt_kernel(const SimtParams p) {
  const int b = blockIdx.x;
  const int hq = blockIdx.y;
  const int h = hq / p.group;
  const int D = p.head_dim;
  const int S = p.page_size;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  __shared__ float q_s[kSimtMaxD];
  __shared__ float w_m[4], w_l[4];
  __shared__ float w_acc[4][kSimtMaxD];

  const T* qrow = static_cast<const T*>(p.q) + static_cast<int64_t>(b) * p.q_stride +
                  static_cast<int64_t>(hq) * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) q_s[d] = to_f32(qrow[d]) * p.scale_log2;
  __syncthreads();

  const int n_pages = clamp_pages(__ldg(p.ctx_lens + b), S, p.bt_stride);
  const int ctx = min(max(__ldg(p.ctx_lens + b), 0), n_pages * S);
  const T* K = static_cast<const T*>(p.k_pool);
  const T* V = static_cast<const T*>(p.v_pool);

  float m = -INFINITY, l = 0.f;
  float acc[kSimtMaxD / 32];
#pragma unroll
  for (int e = 0; e < kSimtMaxD / 32; ++e) acc[e] = 0.f;

  for (int pg = warp; pg < n_pages; pg += 4) {
    int pid = __ldg(p.block_tables + static_cast<int64_t>(b) * p.bt_stride + pg);
    if (pid < 0 || pid >= p.num_pages) {
      if (lane == 0) record_error(p.err, PI_ERR_PAGE_RANGE);
      continue;
    }
    const int64_t tile = (static_cast<int64_t>(pid) * p.hkv + h) * S * D;
    for (int t0 = 0; t0 < S; t0 += 32) {
      const int t = t0 + lane;
      const bool ok = t < S && pg * S + t < ctx;
      float sc = -INFINITY;
      if (ok) {
        const T* kr = K + tile + static_cast<int64_t>(t) * D;
        float dot = 0.f;
        for (int d = 0; d < D; ++d) dot += q_s[d] * to_f32(kr[d]);
        sc = dot;
      }
      float mx = sc;
#pragma unroll
      for (int x = 16; x > 0; x >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, x));
      const float mn = fmaxf(m, mx);
      if (mn == -INFINITY) continue;  // whole chunk masked
      const float al = fast_exp2(m - mn);
      const float pt = ok ? fast_exp2(sc - mn) : 0.f;
      float ps = pt;
#pragma unroll
      for (int x = 16; x > 0; x >>= 1) ps += __shfl_xor_sync(kFull, ps, x);
      l = l * al + ps;
      m = mn;
#pragma unroll
      for (int e = 0; e < kSimtMaxD / 32; ++e) acc[e] *= al;
      const int nt = min(32, S - t0);
      for (int tt = 0; tt < nt; ++tt) {
        const float pv = __shfl_sync(kFull, pt, tt);
        if (pg * S + t0 + tt >= ctx) break;
        const T* vr = V + tile + static_cast<int64_t>(t0 + tt) * D;
#pragma unroll
        for (int e = 0; e < kSimtMaxD / 32; ++e) {
          const int d = lane + 32 * e;
          if (d < D) acc[e] += pv * to_f32(vr[d]);
        }
      }
    }
  }
  if (lane == 0) {
    w_m[warp] = m;
    w_l[warp] = l;
  }
#pragma unroll
  for (int e = 0; e < kSimtMaxD / 32; ++e) {
    const int d = lane + 32 * e;
    if (d < D) w_acc[warp][d] = acc[e];
  }
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < 4; ++w) M = fmaxf(M, w_m[w]);
  float L = 0.f;
  float wt[4];
  for (int w = 0; w < 4; ++w) {
    wt[w] = (w_m[w] == -INFINITY) ? 0.f : fast_exp2(w_m[w] - M);
    L += wt[w] * w_l[w];
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  T* orow = static_cast<T*>(p.out) + static_cast<int64_t>(b) * p.out_stride +
            static_cast<int64_t>(hq) * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float v = 0.f;
    for (int w = 0; w < 4; ++w) v += wt[w] * w_acc[w][d];
    orow[d] = from_f32<T>(v * inv);
  }
}

// ---------------------------------------------------------------------------------
// Host side: tensor-map cache, launch configuration, workspace layout.
// ---------------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
  });
  return fn;
}

struct MapKey {
  const void* ptr;
  uint64_t rows;
  int d;
  int s;
  int dtype;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && d == o.d && s == o.s && dtype == o.dtype;
  }
};

// Encoding a tensor map costs a driver call; decode steps reuse the same pools, so
// keep a small cache keyed on (base, rows, head_dim, page_size, dtype).
bool pool_tensor_map(CUtensorMap* out, const void* base, uint64_t rows, int D, int S, int dtype) {
  constexpr int kCache = 32;
  static std::mutex mu;
  static MapKey keys[kCache];
  static CUtensorMap maps[kCache];
  static int used = 0, next = 0;
  const MapKey key{base, rows, D, S, dtype};
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i) {
    if (keys[i] == key) {
      *out = maps[i];
      return true;
    }
  }
  auto encode = get_encode();
  if (!encode) return false;
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(D) * 2};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(S)};
  cuuint32_t estr[2] = {1u, 1u};
  const CUtensorMapDataType dt =
      dtype == PI_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = encode(&m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  const int slot = used < kCache ? used++ : (next++ % kCache);
  keys[slot] = key;
  maps[slot] = m;
  *out = m;
  return true;
}

struct Layout {
  size_t cnt_off, ml_off, o_off, total;
};

inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Workspace = [arrival counters | partial (m, l) | partial O]. The counter block has
// a fixed size and position whatever the batch shape, so a launch of one shape can
// never find partials of an earlier launch of another shape where its counters are:
// zeroed once, it stays zero because every launch resets the counters it used.
// The last 256 bytes of the block hold the grid-completion counter of the gather
// variant (it also returns to zero at the end of every launch).
constexpr size_t kSegCounterBytes = static_cast<size_t>(kMaxBatch) * kMaxKvHeads * sizeof(int);
constexpr size_t kCounterBytes = kSegCounterBytes + 256;

Layout ws_layout(int head_dim, int sms) {
  Layout L;
  const size_t slots = static_cast<size_t>(sms) * kMaxCtasPerSm * kWarps * 2;
  L.cnt_off = 0;
  L.ml_off = align256(kCounterBytes);
  L.o_off = L.ml_off + align256(slots * kHeadsPad * 2 * sizeof(float));
  L.total = L.o_off + align256(slots * kHeadsPad * static_cast<size_t>(head_dim) * sizeof(float));
  return L;
}

template <typename T, int D, int S, int NS>
int launch_fast_ns(const FastParams& fp, const void* k_pool, const void* v_pool, int64_t rows,
                   int dtype, cudaStream_t stream) {
  if constexpr (fast_smem_bytes<D, S, NS>() > 227 * 1024) {
    // Not even one stage per warp fits with this many warps per CTA.
    return PI_ERR_UNSUPPORTED;
  } else {
  const bool append = fp.slot_mapping != nullptr;
  const bool gather = fp.ag.world > 0;
  const int variant = gather ? 2 : (append ? 1 : 0);
  auto kern = gather ? paged_decode_attn_tma_kernel<T, D, S, NS, false, true>
                     : (append ? paged_decode_attn_tma_kernel<T, D, S, NS, true, false>
                               : paged_decode_attn_tma_kernel<T, D, S, NS, false, false>);
  constexpr size_t smem = fast_smem_bytes<D, S, NS>();
  static int configured_ctas[3][64] = {{0}};  // per variant and device: CTAs per SM (0 = unset)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PI_ERR_CUDA;
  if (dev < 0 || dev >= 64) return PI_ERR_UNSUPPORTED;
  int* configured = &configured_ctas[variant][dev];
  if (*configured == 0) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return PI_ERR_CUDA;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem) != cudaSuccess)
      return PI_ERR_CUDA;
    if (occ < 1) return PI_ERR_UNSUPPORTED;
    *configured = occ < kMaxCtasPerSm ? occ : kMaxCtasPerSm;
  }
  CUtensorMap tk, tv;
  if (!pool_tensor_map(&tk, k_pool, static_cast<uint64_t>(rows), D, S, dtype) ||
      !pool_tensor_map(&tv, v_pool, static_cast<uint64_t>(rows), D, S, dtype))
    return PI_ERR_CUDA;
  const unsigned grid = static_cast<unsigned>(device_sm_count() * *configured);
  return cuda_status(launch_kernel(kern, dim3(grid), dim3(kThreads), smem, stream, tk, tv, fp));
  }
}

// Pipeline depth per launch. Large plain launches use 2 stages per warp, so two CTAs fit
// on an SM: the next launch's CTAs then start while this launch's last CTAs finish (with
// programmatic launch), which measured +2.9% on the 8B decode step. Small launches keep
// the deeper ring and one CTA per SM: twice the warps would cut each (request, head)
// segment into twice the pieces, and on a 1-KV-head shard the extra merges cost 10-15%.
// The host bounds the work by batch x block-table width x KV heads (the context lengths
// are on the device), weighted by the query heads per KV head G, since a page's MMA and
// softmax work grows with G: 600 G-weighted pages per warp at 8 warps per SM separates the
// two regimes. Measured on B200: the 8B batch (G=4, ~120 pages per warp at 8 warps per SM)
// and the 30B-A3B batch (G=8, ~60) run faster on the shallow ring (182.2 vs 186.8 and
// 99.4 vs 103.1 us); KV-head shards of the 8B batch on 2..8 GPUs keep the deep ring.
// pi_set_decode_attn_ring overrides the choice for plain launches.
template <int D, int S>
int ring_stages(int batch, int64_t bt_stride, int hkv, int group, bool plain) {
  constexpr int NS = stages_for<D, S>();
  if constexpr (2 * fast_smem_bytes<D, S, 2>() <= 227 * 1024 && NS > 2) {
    const double pages_bound = static_cast<double>(batch) * static_cast<double>(bt_stride) *
                               static_cast<double>(hkv);
    const double warps2 = static_cast<double>(device_sm_count()) * 2 * kWarps;
    const int ring = decode_attn_ring();
    const bool shallow = ring == PI_ATTN_RING_SHALLOW ||
                         (ring == PI_ATTN_RING_AUTO && pages_bound * group >= 600.0 * warps2);
    if (plain && shallow) return 2;
  }
  return NS;
}

template <typename T, int D, int S>
int launch_fast(const FastParams& fp, const void* k_pool, const void* v_pool, int64_t rows,
                int dtype, cudaStream_t stream) {
  constexpr int NS = stages_for<D, S>();
  const bool plain = fp.slot_mapping == nullptr && fp.ag.world == 0;
  if constexpr (NS > 2) {
    if (ring_stages<D, S>(fp.batch, fp.bt_stride, fp.hkv, fp.group, plain) == 2)
      return launch_fast_ns<T, D, S, 2>(fp, k_pool, v_pool, rows, dtype, stream);
  }
  return launch_fast_ns<T, D, S, NS>(fp, k_pool, v_pool, rows, dtype, stream);
}

// Whether a launch of this shape takes the TMA fast path, pointer alignment aside (the
// dispatcher also needs 16-byte pools and 4-byte q; otherwise it runs the SIMT path).
bool fast_shape(int dtype, int batch, int64_t bt_stride, int num_q_heads, int num_kv_heads,
                int head_dim, int page_size, int64_t num_pages) {
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads != 0) return false;
  const int group = num_q_heads / num_kv_heads;
  const int64_t rows = num_pages * num_kv_heads * page_size;
  const bool half_type = dtype == PI_DTYPE_BF16 || dtype == PI_DTYPE_F16;
  return half_type && (head_dim == 64 || head_dim == 128 || head_dim == 256) &&
         (page_size == 16 || page_size == 32) && group <= kHeadsPad && batch <= kMaxBatch &&
         num_kv_heads <= kMaxKvHeads && rows > 0 && rows < (int64_t{1} << 31) &&
         static_cast<int64_t>(batch) * bt_stride < (int64_t{1} << 31);
}

}  // namespace attn
}  // namespace pi

extern "C" size_t pi_paged_decode_attn_workspace_bytes(int batch, int num_q_heads,
                                                       int num_kv_heads, int head_dim) {
  (void)num_q_heads;
  if (batch <= 0 || num_kv_heads <= 0 || head_dim <= 0) return 0;
  return pi::attn::ws_layout(head_dim, pi::device_sm_count()).total;
}

extern "C" size_t pi_paged_decode_attn_ws_zero_bytes(void) {
  return pi::attn::align256(pi::attn::kCounterBytes);
}

namespace pi {
namespace attn {

// New K/V rows to store before attending (fused append); see FastParams.
struct AppendArgs {
  const void* k_new;
  const void* v_new;
  const int64_t* slot_mapping;
  int64_t new_stride;
};

int attn_dispatch(void* out, const void* q, const void* k_pool, const void* v_pool,
                  const int32_t* block_tables, int64_t bt_stride, const int32_t* ctx_lens,
                  int batch, int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                  int64_t num_pages, float scale, int dtype, int64_t q_stride, int64_t out_stride,
                  void* workspace, size_t workspace_bytes, int* err, cudaStream_t stream,
                  const AppendArgs* app, const pi_peer_gather_t* ag = nullptr) {
  const int eb = elem_bytes_of(dtype);
  if (eb == 0) return PI_ERR_UNSUPPORTED;
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || page_size <= 0 ||
      num_pages < 0 || bt_stride < 0)
    return PI_ERR_BAD_SHAPE;
  if (num_q_heads % num_kv_heads != 0) return PI_ERR_BAD_SHAPE;
  const int64_t row = static_cast<int64_t>(num_q_heads) * head_dim;
  if (q_stride < row || out_stride < row) return PI_ERR_BAD_SHAPE;
  if (batch == 0) return PI_OK;
  if (!out || !q || !k_pool || !v_pool || !block_tables || !ctx_lens) return PI_ERR_NULL_POINTER;
  if (!aligned(block_tables, 4) || !aligned(ctx_lens, 4)) return PI_ERR_MISALIGNED;
  const int group = num_q_heads / num_kv_heads;
  const float scale_log2 = scale * 1.4426950408889634f;
  const int64_t rows = num_pages * num_kv_heads * page_size;

  const bool fast = fast_shape(dtype, batch, bt_stride, num_q_heads, num_kv_heads, head_dim,
                               page_size, num_pages) &&
                    aligned(k_pool, 16) && aligned(v_pool, 16) && aligned(q, 4) &&
                    q_stride % 2 == 0 && aligned(out, 2);
  if (ag != nullptr) {
    if (!fast) return PI_ERR_UNSUPPORTED;  // the peer all-gather lives in the TMA kernel only
    if (ag->world < 1 || ag->world > PI_MAX_PEERS || ag->rank < 0 || ag->rank >= ag->world)
      return PI_ERR_BAD_SHAPE;
    if (ag->rank_stride < static_cast<int64_t>(batch) * out_stride) return PI_ERR_BAD_SHAPE;
    for (int r = 0; r < ag->world; ++r)
      if (ag->peer_out[r] == nullptr || ag->peer_flags[r] == nullptr) return PI_ERR_NULL_POINTER;
    if (static_cast<char*>(ag->peer_out[ag->rank]) + ag->rank * ag->rank_stride * eb !=
        static_cast<char*>(out))
      return PI_ERR_BAD_SHAPE;  // out must be this rank's slice of its gathered buffer
  }
  // The fused append stores whole 16-byte chunks of the new rows.
  const bool fuse = app != nullptr && fast && aligned(app->k_new, 16) &&
                    aligned(app->v_new, 16) && (app->new_stride * eb) % 16 == 0;
  if (app != nullptr && !fuse) {
    // Not fusable: store the rows with the index-copy kernel, then attend.
    const int rc = pi_kv_index_copy(const_cast<void*>(k_pool), const_cast<void*>(v_pool),
                                    app->k_new, app->v_new, app->slot_mapping, batch,
                                    num_kv_heads, head_dim, page_size, num_pages * page_size,
                                    dtype, app->new_stride, err, stream);
    if (rc != PI_OK) return rc;
  }
  if (fast) {
    const Layout L = ws_layout(head_dim, device_sm_count());
    if (workspace == nullptr || workspace_bytes < L.total) return PI_ERR_WORKSPACE;
    if (!aligned(workspace, 256)) return PI_ERR_MISALIGNED;
    FastParams fp;
    fp.out = out;
    fp.q = q;
    fp.block_tables = block_tables;
    fp.ctx_lens = ctx_lens;
    fp.bt_stride = bt_stride;
    fp.q_stride = q_stride;
    fp.out_stride = out_stride;
    fp.num_pages = num_pages;
    fp.batch = batch;
    fp.hkv = num_kv_heads;
    fp.group = group;
    fp.scale_log2 = scale_log2;
    char* ws = static_cast<char*>(workspace);
    fp.ws_cnt = reinterpret_cast<int*>(ws + L.cnt_off);
    fp.ws_ml = reinterpret_cast<float*>(ws + L.ml_off);
    fp.ws_o = reinterpret_cast<float*>(ws + L.o_off);
    fp.err = err;
    fp.k_new = fuse ? app->k_new : nullptr;
    fp.v_new = fuse ? app->v_new : nullptr;
    fp.slot_mapping = fuse ? app->slot_mapping : nullptr;
    fp.new_stride = fuse ? app->new_stride : 0;
    fp.k_pool_w = const_cast<void*>(k_pool);
    fp.v_pool_w = const_cast<void*>(v_pool);
    fp.ag = {};
    fp.ag_done = reinterpret_cast<unsigned*>(ws + L.cnt_off + kSegCounterBytes);
    if (ag != nullptr) {
      // The gather output rows are pushed as 16-byte chunks of whole row groups.
      if ((static_cast<int64_t>(group) * head_dim * eb) % 16 != 0 || (out_stride * eb) % 16 != 0 ||
          (ag->rank_stride * eb) % 16 != 0 ||
          (ag->launch_counter != nullptr && !aligned(ag->launch_counter, 4)))
        return PI_ERR_MISALIGNED;
      fp.ag = *ag;
    }
#define PI_FAST(T, D, S)                                                                  \
  if (head_dim == D && page_size == S)                                                    \
    return launch_fast<T, D, S>(fp, k_pool, v_pool, rows, dtype, stream);
    if (dtype == PI_DTYPE_BF16) {
      PI_FAST(__nv_bfloat16, 64, 16)
      PI_FAST(__nv_bfloat16, 128, 16)
      PI_FAST(__nv_bfloat16, 256, 16)
      PI_FAST(__nv_bfloat16, 64, 32)
      PI_FAST(__nv_bfloat16, 128, 32)
      PI_FAST(__nv_bfloat16, 256, 32)
    } else {
      PI_FAST(__half, 64, 16)
      PI_FAST(__half, 128, 16)
      PI_FAST(__half, 256, 16)
      PI_FAST(__half, 64, 32)
      PI_FAST(__half, 128, 32)
      PI_FAST(__half, 256, 32)
    }
#undef PI_FAST
    return PI_ERR_UNSUPPORTED;
  }

  // Generic SIMT path.
  if (head_dim > kSimtMaxD) return PI_ERR_UNSUPPORTED;
  if (batch > 65535 * 1024 || num_q_heads > 65535) return PI_ERR_UNSUPPORTED;
  if (!aligned(q, eb) || !aligned(out, eb) || !aligned(k_pool, eb) || !aligned(v_pool, eb))
    return PI_ERR_MISALIGNED;
  SimtParams sp;
  sp.out = out;
  sp.q = q;
  sp.k_pool = k_pool;
  sp.v_pool = v_pool;
  sp.block_tables = block_tables;
  sp.ctx_lens = ctx_lens;
  sp.bt_stride = bt_stride;
  sp.q_stride = q_stride;
  sp.out_stride = out_stride;
  sp.num_pages = num_pages;
  sp.hkv = num_kv_heads;
  sp.group = group;
  sp.head_dim = head_dim;
  sp.page_size = page_size;
  sp.scale_log2 = scale_log2;
  sp.err = err;
  const dim3 grid(static_cast<unsigned>(batch), static_cast<unsigned>(num_q_heads));
  if (dtype == PI_DTYPE_F32)
    paged_decode_attn_simt_kernel<float><<<grid, 128, 0, stream>>>(sp);
  else if (dtype == PI_DTYPE_BF16)
    paged_decode_attn_simt_kernel<__nv_bfloat16><<<grid, 128, 0, stream>>>(sp);
  else
    paged_decode_attn_simt_kernel<__half><<<grid, 128, 0, stream>>>(sp);
  return cuda_status(cudaGetLastError());
}

}  // namespace attn
}  // namespace pi

extern "C" int pi_paged_decode_attn_ring_stages(int batch, int64_t bt_stride, int num_q_heads,
                                                int num_kv_heads, int head_dim, int page_size,
                                                int64_t num_pages, int dtype) {
  using namespace pi::attn;
  if (batch <= 0 || bt_stride < 0 || num_pages < 0 ||
      !fast_shape(dtype, batch, bt_stride, num_q_heads, num_kv_heads, head_dim, page_size,
                  num_pages))
    return 0;
#define PI_RING(D, S) \
  if (head_dim == D && page_size == S)                                                        \
    return ring_stages<D, S>(batch, bt_stride, num_kv_heads, num_q_heads / num_kv_heads, true);
  PI_RING(64, 16)
  PI_RING(128, 16)
  PI_RING(256, 16)
  PI_RING(64, 32)
  PI_RING(128, 32)
  PI_RING(256, 32)
#undef PI_RING
  return 0;
}

extern "C" int pi_paged_decode_attn(void* out, const void* q, const void* k_pool,
                                    const void* v_pool, const int32_t* block_tables,
                                    int64_t bt_stride, const int32_t* ctx_lens, int batch,
                                    int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                                    int64_t num_pages, float scale, int dtype, int64_t q_stride,
                                    int64_t out_stride, void* workspace, size_t workspace_bytes,
                                    int* err, cudaStream_t stream) {
  return pi::attn::attn_dispatch(out, q, k_pool, v_pool, block_tables, bt_stride, ctx_lens, batch,
                                 num_q_heads, num_kv_heads, head_dim, page_size, num_pages, scale,
                                 dtype, q_stride, out_stride, workspace, workspace_bytes, err,
                                 stream, nullptr);
}

extern "C" int pi_paged_decode_attn_gather(void* out, const void* q, const void* k_pool,
                                           const void* v_pool, const int32_t* block_tables,
                                           int64_t bt_stride, const int32_t* ctx_lens, int batch,
                                           int num_q_heads, int num_kv_heads, int head_dim,
                                           int page_size, int64_t num_pages, float scale,
                                           int dtype, int64_t q_stride, int64_t out_stride,
                                           void* workspace, size_t workspace_bytes,
                                           const pi_peer_gather_t* gather, int* err,
                                           cudaStream_t stream) {
  if (gather == nullptr) return PI_ERR_NULL_POINTER;
  return pi::attn::attn_dispatch(out, q, k_pool, v_pool, block_tables, bt_stride, ctx_lens, batch,
                                 num_q_heads, num_kv_heads, head_dim, page_size, num_pages, scale,
                                 dtype, q_stride, out_stride, workspace, workspace_bytes, err,
                                 stream, nullptr, gather);
}

extern "C" int pi_paged_decode_attn_append(
    void* out, const void* q, void* k_pool, void* v_pool, const void* k_new, const void* v_new,
    const int64_t* slot_mapping, int64_t new_stride, const int32_t* block_tables,
    int64_t bt_stride, const int32_t* ctx_lens, int batch, int num_q_heads, int num_kv_heads,
    int head_dim, int page_size, int64_t num_pages, float scale, int dtype, int64_t q_stride,
    int64_t out_stride, void* workspace, size_t workspace_bytes, int* err, cudaStream_t stream) {
  using namespace pi;
  if (batch > 0 && (!k_new || !v_new || !slot_mapping)) return PI_ERR_NULL_POINTER;
  if (new_stride < static_cast<int64_t>(num_kv_heads) * head_dim) return PI_ERR_BAD_SHAPE;
  if (slot_mapping && !aligned(slot_mapping, 8)) return PI_ERR_MISALIGNED;
  const attn::AppendArgs app{k_new, v_new, slot_mapping, new_stride};
  return attn::attn_dispatch(out, q, k_pool, v_pool, block_tables, bt_stride, ctx_lens, batch,
                             num_q_heads, num_kv_heads, head_dim, page_size, num_pages, scale,
                             dtype, q_stride, out_stride, workspace, workspace_bytes, err, stream,
                             &app);
}

// ---------------------------------------------------------------------------------
// Allocation-free variant of pi_paged_decode_attn.
//
// Some callers cannot allocate device memory when they run attention: a host loop
// that reaches this library only through the C ABI and owns no CUDA allocator, or
// an engine whose memory planner has already handed every free byte to the page
// pool and the weights, where a cudaMalloc in the middle of decoding would fail or
// stall the device. For them the split-KV scratch (arrival counters and per-warp
// partial results) lives in one fixed array compiled into this library. Every GPU
// that loads the library reserves it until the process exits.
// ---------------------------------------------------------------------------------

namespace pi {
namespace attn {

// Capacity of the built-in scratch: counters (1 MiB) plus partials for
// head_dim <= 128 on a GPU with up to 148 SMs (about 10.9 MB at head_dim 128).
constexpr size_t kStaticScratchBytes = PI_NOALLOC_SCRATCH_BYTES;
static_assert(PI_NOALLOC_SCRATCH_BYTES == (size_t{12} << 20), "header and library agree");

static __device__ __align__(256) unsigned char g_attn_scratch[kStaticScratchBytes];

// Device address of g_attn_scratch on the current device. On the host the symbol
// name is only a handle for the runtime, never an address a kernel may use, so the
// address is looked up once per device (with that device current) and cached.
int static_scratch_address(void** out) {
  static std::mutex mu;
  static void* cached[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PI_ERR_CUDA;
  if (dev < 0 || dev >= 64) return PI_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_scratch) != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();  // do not leave the failure for a later launch check
      return PI_ERR_CUDA;
    }
    cached[dev] = p;
  }
  *out = cached[dev];
  return PI_OK;
}

}  // namespace attn
}  // namespace pi

extern "C" int pi_paged_decode_attn_noalloc(void* out, const void* q, const void* k_pool,
                                            const void* v_pool, const int32_t* block_tables,
                                            int64_t bt_stride, const int32_t* ctx_lens, int batch,
                                            int num_q_heads, int num_kv_heads, int head_dim,
                                            int page_size, int64_t num_pages, float scale,
                                            int dtype, int64_t q_stride, int64_t out_stride,
                                            int* err, cudaStream_t stream) {
  using namespace pi;
  using namespace pi::attn;
  if (batch <= 0 || num_kv_heads <= 0 || head_dim <= 0) {
    // Nothing that needs scratch; let the regular entry point validate and return.
    return pi_paged_decode_attn(out, q, k_pool, v_pool, block_tables, bt_stride, ctx_lens, batch,
                                num_q_heads, num_kv_heads, head_dim, page_size, num_pages, scale,
                                dtype, q_stride, out_stride, nullptr, 0, err, stream);
  }
  if (!fast_shape(dtype, batch, bt_stride, num_q_heads, num_kv_heads, head_dim, page_size,
                  num_pages)) {
    // The generic SIMT path (fp32 pools, other head_dim or page sizes, G > 8, ...)
    // uses no scratch at all: no limit applies.
    return pi_paged_decode_attn(out, q, k_pool, v_pool, block_tables, bt_stride, ctx_lens, batch,
                                num_q_heads, num_kv_heads, head_dim, page_size, num_pages, scale,
                                dtype, q_stride, out_stride, nullptr, 0, err, stream);
  }
  const size_t need =
      pi_paged_decode_attn_workspace_bytes(batch, num_q_heads, num_kv_heads, head_dim);
  if (need > kStaticScratchBytes) return PI_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int st = static_scratch_address(&scratch);
  if (st != PI_OK) return st;
  // The scratch keeps whatever the previous call left; the arrival counters must
  // start at zero, so clear them on the caller's stream (a memset, not an allocation).
  if (cudaMemsetAsync(scratch, 0, pi_paged_decode_attn_ws_zero_bytes(), stream) != cudaSuccess)
    return PI_ERR_CUDA;
  return pi_paged_decode_attn(out, q, k_pool, v_pool, block_tables, bt_stride, ctx_lens, batch,
                              num_q_heads, num_kv_heads, head_dim, page_size, num_pages, scale,
                              dtype, q_stride, out_stride, scratch, kStaticScratchBytes, err,
                              stream);
}
