// Two-SM tcgen05 GEMM for sm_100a: a cluster of two CTAs computes one 256 x 256 output tile
// with tcgen05.mma.cta_group::2. Each CTA stages 128 rows of A and 128 columns of B per stage
// (32 KB instead of the one-SM kernel's 48 KB), so six stages fit where four did, and the pair
// reads each B column once for 256 rows of A. The MMA warp of the even CTA (the leader) issues
// every MMA; each CTA's tensor memory holds its own 128 rows x 256 columns of the accumulator,
// double-buffered, and each CTA's 16 epilogue warps drain their own rows with the same
// four-column epilogue as the one-SM kernel.
//
// Synchronisation inside the pair: both producers' TMA loads complete on the leader's full
// barrier (the leader expects the bytes of both halves); the leader's commits arrive on the
// empty and accumulator-full barriers of both CTAs (one commit per CTA, no multicast); both
// CTAs' epilogue warps arrive on the leader's accumulator-empty barrier. Every mbarrier wait is
// bounded as in the one-SM kernel. No TMA load uses cluster multicast.
//
// A chain runs two GEMMs in one persistent launch when the second reads the first one's output
// rows as its A operand (an MLP block's two linears): the pairs work through a per-pair list of
// tiles of both GEMMs, and a tile of the second waits only for the row block of the first that
// it reads, so neither GEMM's last partial wave leaves SMs idle.
#pragma once
#include "gemm_sm100.cuh"

namespace tgcb_gemm {

#ifndef TGCB_PAIR_STAGES
#define TGCB_PAIR_STAGES 6
#endif
constexpr int P_STAGES = TGCB_PAIR_STAGES;
constexpr int P_A_STAGE = BM * ROW_BYTES;         // 16 KB: this CTA's 128 rows of A
constexpr int P_B_STAGE = (BN / 2) * ROW_BYTES;   // 16 KB: this CTA's 128 columns of B
constexpr int P_SMEM_BYTES = P_STAGES * (P_A_STAGE + P_B_STAGE) + BAR_BYTES + EPI_STAGE_BYTES + 1024;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void bar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// Operand loads carry an L2 evict_last policy (TGCB_LOAD_EVICT_LAST, on unless the source
// defines it 0): a GEMM's operand tiles are read again by the tiles of other pairs, while its
// outputs stream through L2 once; with two 128 MiB outputs (the int8 linear layer) the policy
// keeps the operands from being pushed out by the stores (B200, alternating runs: int8 linear
// 111.4 -> 109.8 us, the training step's forward chain 1.776 -> 1.740 ms, the MLP block's chain
// 213.8 -> 214.1 us).
#ifndef TGCB_LOAD_EVICT_LAST
#define TGCB_LOAD_EVICT_LAST 1
#endif

__device__ __forceinline__ unsigned long long operand_policy() {
  unsigned long long pol = 0;
#if TGCB_LOAD_EVICT_LAST
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
#endif
  return pol;
}

// TMA load into this CTA's shared memory whose completion is counted on `cluster_bar`, which may
// be the peer CTA's barrier (the .cta_group::2 form).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const TgcbTmaDesc* desc, int x, int y, uint32_t cluster_bar,
                                                 unsigned long long pol) {
#if TGCB_LOAD_EVICT_LAST
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<unsigned long long>(desc)), "r"(x), "r"(y), "r"(cluster_bar), "l"(pol)
      : "memory");
#else
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<unsigned long long>(desc)), "r"(x), "r"(y), "r"(cluster_bar)
      : "memory");
#endif
}

template <bool INT8>
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, unsigned long long a, unsigned long long b, uint32_t idesc, uint32_t accumulate) {
  if constexpr (INT8) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8, %5, %6, %7, %8}, p; }" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
  } else {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8, %5, %6, %7, %8}, p; }" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
  }
}

__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const TgcbTmaDesc* desc, int x, int y, int z, uint32_t cluster_bar,
                                                 unsigned long long pol) {
#if TGCB_LOAD_EVICT_LAST
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<unsigned long long>(desc)), "r"(x), "r"(y), "r"(z), "r"(cluster_bar), "l"(pol)
      : "memory");
#else
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<unsigned long long>(desc)), "r"(x), "r"(y), "r"(z), "r"(cluster_bar)
      : "memory");
#endif
}

// Arrive on a barrier (this CTA's or the peer's) when every MMA issued so far has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar) : "memory");
}

// One GEMM run by the pair kernel: C[M,N] = A[M,K] @ B[K,N] and its generated epilogue.
// With SPLIT > 1 the K range is cut into SPLIT equal slices and every (slice, output tile) is
// a work item: item t is slice t / TILES of output tile t % TILES.
template <int M_, int N_, int K_, bool A_MN_, bool B_MN_, class Epi_, int SPLIT_ = 1>
struct PairGemm {
  static constexpr int M = M_;
  static constexpr int N = N_;
  static constexpr int K = K_;
  static constexpr bool A_MN = A_MN_;
  static constexpr bool B_MN = B_MN_;
  static constexpr int SPLIT = SPLIT_;
  using Epi = Epi_;
  static_assert(Epi::VEC4, "the two-SM kernel uses the four-column epilogue");
  static_assert(M % (2 * BM) == 0 && N % BN == 0, "the two-SM kernel covers whole 256 x 256 tiles");
  static constexpr int TILES_M = M / (2 * BM);
  static constexpr int TILES_N = N / BN;
  static constexpr int TILES = TILES_M * TILES_N;  // output tiles
  static constexpr int NUM_TILES = TILES * SPLIT;  // work items
};

// Stands for "no second GEMM" in pair_body.
struct NoGemm {
  static constexpr int NUM_TILES = 0;
  static constexpr int TILES_N = 1;
};

// Stands for "no row prologue" in pair_body. A row prologue (generated) computes the rows of the
// first GEMM's A operand, one warp per row: GROUPS groups of EPI_WARPS rows, row(args, r, lane).
struct NoRows {
  static constexpr int GROUPS = 0;
  static __device__ __forceinline__ void row(const TgcbArgs&, long long, int) {}
};

// The tiles of one GEMM dealt round-robin over the pairs (tile = pair + i * pairs).
template <int NUM_TILES>
struct RoundRobin {
  static __device__ __forceinline__ int count(int pair, int pairs) {
    return pair < NUM_TILES ? (NUM_TILES - 1 - pair) / pairs + 1 : 0;
  }
  static __device__ __forceinline__ int item(int pair, int pairs, int i) { return pair + i * pairs; }
};

// What every role of one CTA needs: shared-memory stages, barriers, tensor memory, its rank.
struct PairCta {
  uint32_t sA, sB, bar0, tmem, rank;
  volatile int* abort_flag;
  __device__ __forceinline__ uint32_t full_bar(int s) const { return bar0 + 8u * s; }
  __device__ __forceinline__ uint32_t empty_bar(int s) const { return bar0 + 8u * (P_STAGES + s); }
  __device__ __forceinline__ uint32_t tfull_bar(int a) const { return bar0 + 8u * (2 * P_STAGES + a); }
  __device__ __forceinline__ uint32_t tempty_bar(int a) const { return bar0 + 8u * (2 * P_STAGES + 2 + a); }
  // chains only (index 2 * P_STAGES + 4 holds the tensor-memory address and the abort flag):
  // the epilogue warps have stored a first-GEMM tile or prologue rows / the signal warp has
  // published them
  __device__ __forceinline__ uint32_t stored_bar(int s) const { return bar0 + 8u * (2 * P_STAGES + 5 + s); }
  __device__ __forceinline__ uint32_t published_bar(int s) const { return bar0 + 8u * (2 * P_STAGES + 7 + s); }
};

// Position in the ring of operand stages (stage, parity) and of the two accumulators.
struct StageRing {
  int stage = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next() {
    if (++stage == P_STAGES) {
      stage = 0;
      phase ^= 1u;
    }
  }
};

struct AccRing {
  int acc = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next() {
    acc ^= 1;
    if (acc == 0) phase ^= 1u;
  }
};

// Producer (one thread per CTA): this CTA's 128 rows of A and 128 columns of B for every
// k-block of one tile, completing on the leader's full barrier.
template <bool INT8, class G>
__device__ __forceinline__ bool produce_tile(const PairCta& c, const TgcbArgs& args, const TgcbTmaDesc* ta,
                                             const TgcbTmaDesc* tb, int tile, StageRing& r) {
  constexpr int EB = INT8 ? 1 : 4;
  constexpr int KB = ROW_BYTES / EB;
  constexpr int NUM_KB = (G::K + KB - 1) / KB;
  constexpr int KB_PER = NUM_KB / G::SPLIT;  // k-blocks of one item
  static_assert(NUM_KB % G::SPLIT == 0, "K splits into whole k-blocks");
  constexpr uint32_t PAIR_TX = 2 * (P_A_STAGE + P_B_STAGE);  // both CTAs' halves land on the leader's barrier
  const int out = tile % G::TILES;
  const int kb0 = (tile / G::TILES) * KB_PER;
  const int tm = out / G::TILES_N;
  const int tn = out % G::TILES_N;
  const int arow = tm * 2 * BM + (int)c.rank * BM;      // this CTA's rows of A
  const int bcol = tn * BN + (int)c.rank * (BN / 2);    // this CTA's columns of B
  const unsigned long long pol = operand_policy();
  for (int kb = kb0; kb < kb0 + KB_PER; ++kb) {
    if (!bar_wait(c.empty_bar(r.stage), r.phase ^ 1u, c.abort_flag, args.status, TGCB_STATUS_TIMEOUT_PRODUCER)) return false;
    const uint32_t lead_full = cluster_addr(c.full_bar(r.stage), 0);
    if (c.rank == 0) bar_arrive_expect(c.full_bar(r.stage), PAIR_TX);
    const uint32_t a_dst = c.sA + r.stage * P_A_STAGE;
    const uint32_t b_dst = c.sB + r.stage * P_B_STAGE;
    if (!G::A_MN) {
      tma_load_2d_pair(a_dst, ta, kb * KB, arow, lead_full, pol);
    } else if constexpr (chunked_mn(INT8, G::A_MN, G::M)) {
      tma_load_3d_pair(a_dst, ta, 0, kb * KB, arow / 32, lead_full, pol);
    } else {
#pragma unroll
      for (int q = 0; q < BM * EB / ROW_BYTES; ++q)
        tma_load_2d_pair(a_dst + q * (KB * ROW_BYTES), ta, arow + q * (ROW_BYTES / EB), kb * KB, lead_full, pol);
    }
    if (!G::B_MN) {
      tma_load_2d_pair(b_dst, tb, kb * KB, bcol, lead_full, pol);
    } else if constexpr (chunked_mn(INT8, G::B_MN, G::N)) {
      tma_load_3d_pair(b_dst, tb, 0, kb * KB, bcol / 32, lead_full, pol);
    } else {
#pragma unroll
      for (int q = 0; q < (BN / 2) * EB / ROW_BYTES; ++q)
        tma_load_2d_pair(b_dst + q * (KB * ROW_BYTES), tb, bcol + q * (ROW_BYTES / EB), kb * KB, lead_full, pol);
    }
    r.next();
  }
  return true;
}

// MMA issue (one thread of the leader): one 256 x 256 tile into accumulator a.acc, then
// commits that make both CTAs' accumulator-full barriers complete when the tile is done.
template <bool INT8, class G>
__device__ __forceinline__ bool mma_tile(const PairCta& c, const TgcbArgs& args, StageRing& r, AccRing& a) {
  constexpr int EB = INT8 ? 1 : 4;
  constexpr int KB = ROW_BYTES / EB;
  constexpr int MMA_K = 32 / EB;
  constexpr int KSTEPS = KB / MMA_K;
  constexpr int NUM_KB = (G::K + KB - 1) / KB;
  constexpr uint32_t MN_LAYOUT = INT8 ? 2u : 1u;
  constexpr uint32_t MN_SBO = INT8 ? 1024u : 512u;
  // Instruction descriptor as in the one-SM kernel, with M = 256 (the pair's rows).
  constexpr uint32_t IDESC = (INT8 ? (2u << 4) : (1u << 4)) | (INT8 ? (1u << 7) : (2u << 7)) |
                             (INT8 ? (1u << 10) : (2u << 10)) | ((G::A_MN ? 1u : 0u) << 15) |
                             ((G::B_MN ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)((2 * BM) >> 4) << 24);
  constexpr int KB_PER = NUM_KB / G::SPLIT;  // k-blocks of one item
  if (!bar_wait(c.tempty_bar(a.acc), a.phase ^ 1u, c.abort_flag, args.status, TGCB_STATUS_TIMEOUT_MMA)) return false;
  tc_fence_after();
  const uint32_t d = c.tmem + (uint32_t)(a.acc * BN);
  for (int kb = 0; kb < KB_PER; ++kb) {
    if (!bar_wait(c.full_bar(r.stage), r.phase, c.abort_flag, args.status, TGCB_STATUS_TIMEOUT_MMA)) return false;
    tc_fence_after();
    const uint32_t a_base = c.sA + r.stage * P_A_STAGE;
    const uint32_t b_base = c.sB + r.stage * P_B_STAGE;
#pragma unroll
    for (int k = 0; k < KSTEPS; ++k) {
      const unsigned long long adesc = G::A_MN ? umma_desc(a_base + k * MMA_K * ROW_BYTES, KB * ROW_BYTES, MN_SBO, MN_LAYOUT)
                                               : umma_desc(a_base + k * 32, 16, 1024);
      const unsigned long long bdesc = G::B_MN ? umma_desc(b_base + k * MMA_K * ROW_BYTES, KB * ROW_BYTES, MN_SBO, MN_LAYOUT)
                                               : umma_desc(b_base + k * 32, 16, 1024);
      mma_pair<INT8>(d, adesc, bdesc, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
    }
    mma_commit_pair(cluster_addr(c.empty_bar(r.stage), 0));
    mma_commit_pair(cluster_addr(c.empty_bar(r.stage), 1));
    r.next();
  }
  mma_commit_pair(cluster_addr(c.tfull_bar(a.acc), 0));
  mma_commit_pair(cluster_addr(c.tfull_bar(a.acc), 1));
  a.next();
  return true;
}

// Epilogue (one warp): its 32 rows x 64 columns of this CTA's half of a tile, 8 columns at a
// time out of tensor memory, transposed through shared memory so that two lanes hand one
// row's four consecutive columns to the generated apply4; then the accumulator goes back to
// the leader.
//
// A K-split item (G::SPLIT > 1) stores its partial accumulator instead, as slice s of the
// workspace ws[SPLIT][M][N] (32-bit: float, or int for int8), and counts it in its region's
// counter (region = CTA rank, lane quadrant and column quarter: the 32 x 64 block this warp
// covers in every slice). The warp that counts the last slice of a region sums the SPLIT
// partials of the region in slice order 0, 1, ... (the same order whichever slice finished
// last) and runs apply4 on the sums: the result does not depend on timing.
template <bool INT8, class G>
__device__ __forceinline__ bool epilogue_tile(const PairCta& c, const TgcbArgs& args, int tile, AccRing& a, uint4* st4,
                                              int quad, int cbase, int lane, uint32_t lead_tempty0, uint32_t lead_tempty1,
                                              void* ws, unsigned* counters) {
  using Epi = typename G::Epi;
  constexpr int C8 = BN / 4 / 8;
  constexpr bool SPLIT = G::SPLIT > 1;
  const int out = tile % G::TILES;
  const int tm = out / G::TILES_N;
  const int tn = out % G::TILES_N;
  const long long row0 = (long long)tm * 2 * BM + (long long)c.rank * BM + quad * 32;
  typename Epi::Loads4 cur[2], nxt[2];
  if constexpr (!SPLIT) {
#pragma unroll
    for (int it = 0; it < 2; ++it)
      cur[it] = Epi::load4(args, row0 + 16 * it + (lane >> 1), (long long)tn * BN + cbase + 4 * (lane & 1));
  }
  bool ok = true;
  if (lane == 0) ok = bar_wait(c.tfull_bar(a.acc), a.phase, c.abort_flag, args.status, TGCB_STATUS_TIMEOUT_EPILOGUE);
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  if (!ok) return false;
  tc_fence_after();
  uint4* slice = nullptr;
  if constexpr (SPLIT) slice = reinterpret_cast<uint4*>(static_cast<uint32_t*>(ws) + (long long)(tile / G::TILES) * G::M * G::N);
#pragma unroll 1
  for (int q = 0; q < C8; ++q) {
    uint32_t v8[8];
    tmem_ld8(c.tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(a.acc * BN + cbase + q * 8), v8);
    st4[lane * 2 + (0 ^ ((lane >> 2) & 1))] = make_uint4(v8[0], v8[1], v8[2], v8[3]);
    st4[lane * 2 + (1 ^ ((lane >> 2) & 1))] = make_uint4(v8[4], v8[5], v8[6], v8[7]);
    __syncwarp();
    const long long col0 = (long long)tn * BN + cbase + q * 8;
    if constexpr (!SPLIT) {
      if (q + 1 < C8) {
#pragma unroll
        for (int it = 0; it < 2; ++it) nxt[it] = Epi::load4(args, row0 + 16 * it + (lane >> 1), col0 + 8 + 4 * (lane & 1));
      }
    }
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int rr = 16 * it + (lane >> 1);
      const int qq = lane & 1;
      const uint4 v = st4[rr * 2 + (qq ^ ((rr >> 2) & 1))];
      if constexpr (SPLIT) {
        slice[((row0 + rr) * G::N + col0 + 4 * qq) >> 2] = v;  // the raw partial accumulator
      } else if constexpr (INT8) {
        Epi::apply4(args, row0 + rr, col0 + 4 * qq, make_int4((int)v.x, (int)v.y, (int)v.z, (int)v.w), cur[it]);
      } else {
        Epi::apply4(args, row0 + rr, col0 + 4 * qq,
                    make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w)),
                    cur[it]);
      }
    }
    __syncwarp();
    if constexpr (!SPLIT) {
#pragma unroll
      for (int it = 0; it < 2; ++it) cur[it] = nxt[it];
    }
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) bar_arrive_cluster(a.acc == 0 ? lead_tempty0 : lead_tempty1);
  a.next();
  if constexpr (SPLIT) {
    // publish this slice of the region; the last of the SPLIT slices finishes the region
    __threadfence();
    __syncwarp();
    unsigned seen = 0;
    if (lane == 0) seen = atomicAdd(counters + out * 32 + (int)c.rank * 16 + (cbase / (BN / 4)) * 4 + quad, 1u);
    seen = __shfl_sync(0xffffffffu, seen, 0);
    if (seen == (unsigned)(G::SPLIT - 1)) {
      __threadfence();
      const uint4* base = reinterpret_cast<const uint4*>(ws);
      constexpr long long SLICE = (long long)G::M * G::N / 4;
#pragma unroll 1
      for (int q = 0; q < C8; ++q) {
        const long long col0 = (long long)tn * BN + cbase + q * 8;
#pragma unroll
        for (int it = 0; it < 2; ++it) {
          const long long row = row0 + 16 * it + (lane >> 1);
          const long long col = col0 + 4 * (lane & 1);
          const long long e = (row * G::N + col) >> 2;
          uint4 v = __ldcg(base + e);
          if constexpr (INT8) {
            int4 t = make_int4((int)v.x, (int)v.y, (int)v.z, (int)v.w);
            for (int k = 1; k < G::SPLIT; ++k) {
              const uint4 w = __ldcg(base + k * SLICE + e);
              t.x += (int)w.x;
              t.y += (int)w.y;
              t.z += (int)w.z;
              t.w += (int)w.w;
            }
            Epi::apply4(args, row, col, t, Epi::load4(args, row, col));
          } else {
            float4 t = make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
            for (int k = 1; k < G::SPLIT; ++k) {
              const uint4 w = __ldcg(base + k * SLICE + e);
              t.x = __fadd_rn(t.x, __uint_as_float(w.x));
              t.y = __fadd_rn(t.y, __uint_as_float(w.y));
              t.z = __fadd_rn(t.z, __uint_as_float(w.z));
              t.w = __fadd_rn(t.w, __uint_as_float(w.w));
            }
            Epi::apply4(args, row, col, t, Epi::load4(args, row, col));
          }
        }
      }
    }
  }
  return true;
}

// Bounded wait until *count reaches target (acquire at GPU scope), then a proxy fence so that
// this thread's later TMA loads see what the counted writers stored. Gives up when the CTA
// aborts, when any CTA has recorded a failure, or after the wall-clock budget.
__device__ __forceinline__ bool wait_count(const unsigned* count, unsigned target, volatile int* abort_flag, int* status) {
  unsigned long long start = 0;
  for (uint32_t it = 0;; ++it) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(count) : "memory");
    if (v >= target) {
      asm volatile("fence.proxy.async.global;" ::: "memory");
      return true;
    }
    if (*abort_flag || *reinterpret_cast<volatile int*>(status) != TGCB_STATUS_OK) return false;
    __nanosleep(128);
    if ((it & 63u) == 63u) {
      const unsigned long long t = now_ns();
      if (start == 0) {
        start = t;
      } else if (t - start > WAIT_BUDGET_NS) {
        *abort_flag = 1;
        tgcb_fail(status, TGCB_STATUS_TIMEOUT_PRODUCER);
        return false;
      }
    }
  }
}

// Epilogue side of the ev-th publish event of a CTA (one call per epilogue warp, after the
// warp's stores): wait until the signal warp has published the event that used this barrier
// slot two events ago, then arrive on the slot's stored barrier (release, CTA scope).
__device__ __forceinline__ bool hand_over(const PairCta& c, const TgcbArgs& args, int ev, int lane) {
  __syncwarp();
  bool ok = true;
  if (lane == 0 && ev >= 2)
    ok = bar_wait(c.published_bar(ev & 1), (uint32_t)(((ev >> 1) - 1) & 1), c.abort_flag, args.status,
                  TGCB_STATUS_TIMEOUT_EPILOGUE);
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  if (ok && lane == 0) bar_arrive(c.stored_bar(ev & 1));
  return ok;
}

// Signal side of the ev-th publish event: once every epilogue warp has arrived, add 1 to
// *counter (release, GPU scope: the warps' stores become visible to an acquiring reader on
// any SM) and free the barrier slot.
__device__ __forceinline__ bool publish(const PairCta& c, const TgcbArgs& args, int ev, unsigned* counter) {
  if (!bar_wait(c.stored_bar(ev & 1), (uint32_t)((ev >> 1) & 1), c.abort_flag, args.status, TGCB_STATUS_TIMEOUT_EPILOGUE))
    return false;
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
  bar_arrive(c.published_bar(ev & 1));
  return true;
}

// Threads of a chain CTA: one more warp, which publishes stored rows.
constexpr int CHAIN_THREADS = THREADS + 32;

// The pair kernel. Sched lists each pair's work items; item t < G1::NUM_TILES is tile t of
// G1, item G1::NUM_TILES + t tile t of G2. With a second GEMM (a chain), G2 reads G1's output
// as its A operand. When the 16 epilogue warps of a CTA have stored their rows of a G1 tile
// they arrive on a stored barrier (release, CTA scope) and go on; the signal warp waits there
// and adds 1 to rows_done[row block] (release, GPU scope), so no epilogue warp waits for its
// stores to drain. A producer loads A for a G2 tile of row block m only after rows_done[m]
// holds G1::TILES_N * 2 (every tile of the block, both CTAs; acquire + proxy fence). The
// stored and published barriers are double-buffered, so the epilogue runs at most two G1
// tiles ahead of the signal warp.
//
// With a row prologue (Pro), G1's A operand is itself computed in this launch: before their
// first tile the epilogue warps of CTA b compute row groups b, b + gridDim.x, ... (one row per
// warp, Pro::row), each published like a G1 tile into rows_ready[row block] (rows_done +
// G1::TILES_M), and a producer loads A for a G1 tile of row block m only after all
// 2 * BM / EPI_WARPS groups of the block are counted.
//
// The counters hold zeros when the kernel starts. Every pair must be resident at once for the
// waits to end; the runtime checks that before the first chain launch, and the waits are
// bounded all the same.
template <bool INT8, class G1, class G2, class Sched, class Pro = NoRows>
__device__ __forceinline__ void pair_body(const TgcbArgs& args, const TgcbTmaDesc* ta1, const TgcbTmaDesc* tb1,
                                          const TgcbTmaDesc* ta2, const TgcbTmaDesc* tb2, unsigned* rows_done,
                                          void* ws = nullptr) {
  constexpr bool CHAIN = G2::NUM_TILES > 0;
  constexpr bool PRO = Pro::GROUPS > 0;
  constexpr bool SIGNAL = CHAIN || PRO;  // a signal warp publishes stored rows
  constexpr unsigned ROW_COUNT = (unsigned)G1::TILES_N * 2u;
  constexpr unsigned GROUP_COUNT = (unsigned)(2 * BM / EPI_WARPS);  // row groups per 256-row block
  constexpr int NTHREADS = SIGNAL ? CHAIN_THREADS : THREADS;
  static_assert(!PRO || Pro::GROUPS * EPI_WARPS == G1::M, "a row prologue computes every row of G1's A");
  unsigned* rows_ready = rows_done + G1::TILES_M;

  extern __shared__ unsigned char tgcb_smem_raw[];
  const uint32_t raw = smem_addr(tgcb_smem_raw);
  unsigned char* smem = tgcb_smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  PairCta c;
  c.sA = smem_addr(smem);
  c.sB = c.sA + P_STAGES * P_A_STAGE;
  unsigned long long* bars = reinterpret_cast<unsigned long long*>(smem + P_STAGES * (P_A_STAGE + P_B_STAGE));
  c.bar0 = smem_addr(bars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * P_STAGES + 4);
  c.abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  c.rank = cluster_rank();  // 0: the leader, which issues the MMAs
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;

  if (blockDim.x != NTHREADS || (gridDim.x & 1u) != 0u) {
    // both CTAs of every pair see the same launch shape, so both leave here together
    if (threadIdx.x == 0) tgcb_fail(args.status, TGCB_STATUS_BAD_LAUNCH);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      bar_init(c.full_bar(s), 1);
      bar_init(c.empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      bar_init(c.tfull_bar(a), 1);
      bar_init(c.tempty_bar(a), 2 * EPI_WARPS);
      if (SIGNAL) {
        bar_init(c.stored_bar(a), EPI_WARPS);
        bar_init(c.published_bar(a), 1);
      }
    }
    *c.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    // both CTAs' warp 1 allocate together; the same address comes back in both
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"((uint32_t)TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers are initialised before anything signals them
  tc_fence_after();
  c.tmem = *tmem_slot;
  const int items = Sched::count(pair, pairs);

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(ta1)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(tb1)) : "memory");
      if constexpr (CHAIN) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(ta2)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(tb2)) : "memory");
      }
      StageRing r;
      for (int i = 0; i < items; ++i) {
        const int t = Sched::item(pair, pairs, i);
        bool ok = false;
        if (CHAIN && t >= G1::NUM_TILES) {
          if constexpr (CHAIN) {
            const int t2 = t - G1::NUM_TILES;
            ok = wait_count(rows_done + t2 / G2::TILES_N, ROW_COUNT, c.abort_flag, args.status) &&
                 produce_tile<INT8, G2>(c, args, ta2, tb2, t2, r);
          }
        } else {
          ok = (!PRO || wait_count(rows_ready + t / G1::TILES_N, GROUP_COUNT, c.abort_flag, args.status)) &&
               produce_tile<INT8, G1>(c, args, ta1, tb1, t, r);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && c.rank == 0) {
      StageRing r;
      AccRing a;
      for (int i = 0; i < items; ++i) {
        const int t = Sched::item(pair, pairs, i);
        bool ok = false;
        if (CHAIN && t >= G1::NUM_TILES) {
          if constexpr (CHAIN) ok = mma_tile<INT8, G2>(c, args, r, a);
        } else {
          ok = mma_tile<INT8, G1>(c, args, r, a);
        }
        if (!ok) break;
      }
    }
  } else if (warp < 2 + EPI_WARPS) {
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int cbase = (ew >> 2) * (BN / 4);
    uint4* st4 = reinterpret_cast<uint4*>(reinterpret_cast<uint32_t*>(smem + P_STAGES * (P_A_STAGE + P_B_STAGE) + BAR_BYTES) +
                                          ew * STAGE_WORDS);
    const uint32_t lead_tempty0 = cluster_addr(c.tempty_bar(0), 0);
    const uint32_t lead_tempty1 = cluster_addr(c.tempty_bar(1), 0);
    AccRing a;
    int ev = 0;  // stores this warp has handed to the signal warp
    bool ok = true;
    if constexpr (PRO) {
      for (int q = blockIdx.x; q < Pro::GROUPS; q += gridDim.x) {
        Pro::row(args, (long long)q * EPI_WARPS + ew, lane);
        if (!(ok = hand_over(c, args, ev++, lane))) break;
      }
    }
    for (int i = 0; ok && i < items; ++i) {
      const int t = Sched::item(pair, pairs, i);
      if (CHAIN && t >= G1::NUM_TILES) {
        if constexpr (CHAIN) {
          if (!epilogue_tile<INT8, G2>(c, args, t - G1::NUM_TILES, a, st4, quad, cbase, lane, lead_tempty0, lead_tempty1, ws,
                                      rows_done)) break;
        }
      } else {
        if (!epilogue_tile<INT8, G1>(c, args, t, a, st4, quad, cbase, lane, lead_tempty0, lead_tempty1, ws, rows_done)) break;
        if constexpr (CHAIN) ok = hand_over(c, args, ev++, lane);  // this warp's rows of the tile are stored
      }
    }
  } else if constexpr (SIGNAL) {
    // the signal warp: for each row group of the prologue and each first-GEMM tile of this
    // CTA, once the epilogue warps have stored it, count it for the producers of every pair
    if (lane == 0) {
      int ev = 0;
      bool ok = true;
      if constexpr (PRO) {
        for (int q = blockIdx.x; ok && q < Pro::GROUPS; q += gridDim.x)
          ok = publish(c, args, ev++, rows_ready + q * EPI_WARPS / (2 * BM));
      }
      if constexpr (CHAIN) {
        for (int i = 0; ok && i < items; ++i) {
          const int t = Sched::item(pair, pairs, i);
          if (t < G1::NUM_TILES) ok = publish(c, args, ev++, rows_done + t / G1::TILES_N);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA frees its tensor memory or leaves while the pair still uses it
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(c.tmem), "r"((uint32_t)TMEM_COLS));
  }
}

// One GEMM on SM pairs.
template <int M, int N, int K, bool INT8, bool A_MN, bool B_MN, class Epi>
__device__ __forceinline__ void gemm_body_pair(const TgcbArgs& args, const TgcbTmaDesc* ta, const TgcbTmaDesc* tb) {
  using G = PairGemm<M, N, K, A_MN, B_MN, Epi>;
  pair_body<INT8, G, NoGemm, RoundRobin<G::NUM_TILES>>(args, ta, tb, ta, tb, nullptr);
}

// One GEMM on SM pairs with K cut into SPLIT slices (for GEMMs with fewer output tiles than
// pairs): ws holds SPLIT x M x N partials, counters one zeroed word per 32 x 64 region of every
// output tile (TILES x 32), both in the arena.
template <int M, int N, int K, bool INT8, bool A_MN, bool B_MN, class Epi, int SPLIT>
__device__ __forceinline__ void gemm_split_pair(const TgcbArgs& args, const TgcbTmaDesc* ta, const TgcbTmaDesc* tb,
                                                void* ws, unsigned* counters) {
  using G = PairGemm<M, N, K, A_MN, B_MN, Epi, SPLIT>;
  pair_body<INT8, G, NoGemm, RoundRobin<G::NUM_TILES>>(args, ta, tb, ta, tb, counters, ws);
}

// Two GEMMs on SM pairs, the second reading the first's output as A, in one persistent launch.
// With Pro, the rows of the first GEMM's A operand are computed in the same launch. `counters`
// holds G1::TILES_M words for the second GEMM's waits, then (with Pro) as many for the first's.
template <bool INT8, class G1, class G2, class Sched, class Pro = NoRows>
__device__ __forceinline__ void gemm_chain_pair(const TgcbArgs& args, const TgcbTmaDesc* ta1, const TgcbTmaDesc* tb1,
                                                const TgcbTmaDesc* ta2, const TgcbTmaDesc* tb2, unsigned* counters) {
  static_assert(G1::M == G2::M && !G2::A_MN, "a chain's second GEMM reads the first one's rows as its A");
  static_assert(Pro::GROUPS == 0 || !G1::A_MN, "a row prologue writes the rows of a K-major A");
  if (gridDim.x != 2u * Sched::PAIRS) {
    if (threadIdx.x == 0) tgcb_fail(args.status, TGCB_STATUS_BAD_LAUNCH);
    return;
  }
  pair_body<INT8, G1, G2, Sched, Pro>(args, ta1, tb1, ta2, tb2, counters);
}

}  // namespace tgcb_gemm
