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
#pragma once
#include "gemm_sm100.cuh"

namespace tgcb_gemm {

constexpr int P_STAGES = 6;
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

// TMA load into this CTA's shared memory whose completion is counted on `cluster_bar`, which may
// be the peer CTA's barrier (the .cta_group::2 form).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const TgcbTmaDesc* desc, int x, int y, uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<unsigned long long>(desc)), "r"(x), "r"(y), "r"(cluster_bar)
      : "memory");
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

// Arrive on a barrier (this CTA's or the peer's) when every MMA issued so far has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar) : "memory");
}

template <int M, int N, int K, bool INT8, bool A_MN, bool B_MN, class Epi>
__device__ __forceinline__ void gemm_body_pair(const TgcbArgs& args, const TgcbTmaDesc* ta, const TgcbTmaDesc* tb) {
  static_assert(Epi::VEC4, "the two-SM kernel uses the four-column epilogue");
  static_assert(M % (2 * BM) == 0 && N % BN == 0, "the two-SM kernel covers whole 256 x 256 tiles");
  constexpr int EB = INT8 ? 1 : 4;
  constexpr int KB = ROW_BYTES / EB;
  constexpr int MMA_K = 32 / EB;
  constexpr int KSTEPS = KB / MMA_K;
  constexpr int NUM_KB = (K + KB - 1) / KB;
  constexpr int TILES_M = M / (2 * BM);
  constexpr int TILES_N = N / BN;
  constexpr int NUM_TILES = TILES_M * TILES_N;
  constexpr uint32_t PAIR_TX = 2 * (P_A_STAGE + P_B_STAGE);  // both CTAs' halves land on the leader's barrier
  constexpr uint32_t MN_LAYOUT = INT8 ? 2u : 1u;
  constexpr uint32_t MN_SBO = INT8 ? 1024u : 512u;
  // Instruction descriptor as in the one-SM kernel, with M = 256 (the pair's rows).
  constexpr uint32_t IDESC = (INT8 ? (2u << 4) : (1u << 4)) | (INT8 ? (1u << 7) : (2u << 7)) |
                             (INT8 ? (1u << 10) : (2u << 10)) | ((A_MN ? 1u : 0u) << 15) | ((B_MN ? 1u : 0u) << 16) |
                             ((uint32_t)(BN >> 3) << 17) | ((uint32_t)((2 * BM) >> 4) << 24);

  extern __shared__ unsigned char tgcb_smem_raw[];
  const uint32_t raw = smem_addr(tgcb_smem_raw);
  unsigned char* smem = tgcb_smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  const uint32_t sA = smem_addr(smem);
  const uint32_t sB = sA + P_STAGES * P_A_STAGE;
  unsigned long long* bars = reinterpret_cast<unsigned long long*>(smem + P_STAGES * (P_A_STAGE + P_B_STAGE));
  const uint32_t bar0 = smem_addr(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (P_STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * P_STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * P_STAGES + 2 + a); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * P_STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0: the leader, which issues the MMAs
  const uint32_t peer = rank ^ 1u;
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;

  if (blockDim.x != THREADS || (gridDim.x & 1u) != 0u) {
    // both CTAs of every pair see the same launch shape, so both leave here together
    if (threadIdx.x == 0) tgcb_fail(args.status, TGCB_STATUS_BAD_LAUNCH);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      bar_init(full_bar(s), 1);
      bar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      bar_init(tfull_bar(a), 1);
      bar_init(tempty_bar(a), 2 * EPI_WARPS);
    }
    *abort_flag = 0;
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
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(ta)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(tb)) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = pair; tile < NUM_TILES; tile += pairs) {
        const int tm = tile / TILES_N;
        const int tn = tile % TILES_N;
        const int arow = tm * 2 * BM + (int)rank * BM;      // this CTA's rows of A
        const int bcol = tn * BN + (int)rank * (BN / 2);    // this CTA's columns of B
        for (int kb = 0; kb < NUM_KB; ++kb) {
          if (!bar_wait(empty_bar(stage), phase ^ 1u, abort_flag, args.status, TGCB_STATUS_TIMEOUT_PRODUCER)) goto producer_done;
          const uint32_t lead_full = cluster_addr(full_bar(stage), 0);
          if (rank == 0) bar_arrive_expect(full_bar(stage), PAIR_TX);
          const uint32_t a_dst = sA + stage * P_A_STAGE;
          const uint32_t b_dst = sB + stage * P_B_STAGE;
          if (!A_MN) {
            tma_load_2d_pair(a_dst, ta, kb * KB, arow, lead_full);
          } else {
#pragma unroll
            for (int c = 0; c < BM * EB / ROW_BYTES; ++c)
              tma_load_2d_pair(a_dst + c * (KB * ROW_BYTES), ta, arow + c * (ROW_BYTES / EB), kb * KB, lead_full);
          }
          if (!B_MN) {
            tma_load_2d_pair(b_dst, tb, kb * KB, bcol, lead_full);
          } else {
#pragma unroll
            for (int c = 0; c < (BN / 2) * EB / ROW_BYTES; ++c)
              tma_load_2d_pair(b_dst + c * (KB * ROW_BYTES), tb, bcol + c * (ROW_BYTES / EB), kb * KB, lead_full);
          }
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = pair; tile < NUM_TILES; tile += pairs) {
        if (!bar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_flag, args.status, TGCB_STATUS_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < NUM_KB; ++kb) {
          if (!bar_wait(full_bar(stage), phase, abort_flag, args.status, TGCB_STATUS_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = sA + stage * P_A_STAGE;
          const uint32_t b_base = sB + stage * P_B_STAGE;
#pragma unroll
          for (int k = 0; k < KSTEPS; ++k) {
            const unsigned long long adesc = A_MN ? umma_desc(a_base + k * MMA_K * ROW_BYTES, KB * ROW_BYTES, MN_SBO, MN_LAYOUT)
                                                  : umma_desc(a_base + k * 32, 16, 1024);
            const unsigned long long bdesc = B_MN ? umma_desc(b_base + k * MMA_K * ROW_BYTES, KB * ROW_BYTES, MN_SBO, MN_LAYOUT)
                                                  : umma_desc(b_base + k * 32, 16, 1024);
            mma_pair<INT8>(d, adesc, bdesc, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit_pair(cluster_addr(empty_bar(stage), 0));
          mma_commit_pair(cluster_addr(empty_bar(stage), 1));
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit_pair(cluster_addr(tfull_bar(acc), 0));
        mma_commit_pair(cluster_addr(tfull_bar(acc), 1));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int part = ew >> 2;
    uint32_t* stage = reinterpret_cast<uint32_t*>(smem + P_STAGES * (P_A_STAGE + P_B_STAGE) + BAR_BYTES) + ew * STAGE_WORDS;
    uint4* st4 = reinterpret_cast<uint4*>(stage);
    const uint32_t lead_tempty0 = cluster_addr(tempty_bar(0), 0);
    const uint32_t lead_tempty1 = cluster_addr(tempty_bar(1), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    constexpr int C8 = BN / 4 / 8;
    const int cbase = part * (BN / 4);
    for (int tile = pair; tile < NUM_TILES; tile += pairs) {
      const int tm = tile / TILES_N;
      const int tn = tile % TILES_N;
      const long long row0 = (long long)tm * 2 * BM + (long long)rank * BM + quad * 32;
      typename Epi::Loads4 cur[2], nxt[2];
#pragma unroll
      for (int it = 0; it < 2; ++it)
        cur[it] = Epi::load4(args, row0 + 16 * it + (lane >> 1), (long long)tn * BN + cbase + 4 * (lane & 1));
      bool ok = true;
      if (lane == 0) ok = bar_wait(tfull_bar(acc), acc_phase, abort_flag, args.status, TGCB_STATUS_TIMEOUT_EPILOGUE);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < C8; ++c) {
        uint32_t r[8];
        tmem_ld8(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN + cbase + c * 8), r);
        st4[lane * 2 + (0 ^ ((lane >> 2) & 1))] = make_uint4(r[0], r[1], r[2], r[3]);
        st4[lane * 2 + (1 ^ ((lane >> 2) & 1))] = make_uint4(r[4], r[5], r[6], r[7]);
        __syncwarp();
        const long long col0 = (long long)tn * BN + cbase + c * 8;
        if (c + 1 < C8) {
#pragma unroll
          for (int it = 0; it < 2; ++it) nxt[it] = Epi::load4(args, row0 + 16 * it + (lane >> 1), col0 + 8 + 4 * (lane & 1));
        }
#pragma unroll
        for (int it = 0; it < 2; ++it) {
          const int rr = 16 * it + (lane >> 1);
          const int qq = lane & 1;
          const uint4 v = st4[rr * 2 + (qq ^ ((rr >> 2) & 1))];
          if constexpr (INT8) {
            Epi::apply4(args, row0 + rr, col0 + 4 * qq, make_int4((int)v.x, (int)v.y, (int)v.z, (int)v.w), cur[it]);
          } else {
            Epi::apply4(args, row0 + rr, col0 + 4 * qq,
                        make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w)),
                        cur[it]);
          }
        }
        __syncwarp();
#pragma unroll
        for (int it = 0; it < 2; ++it) cur[it] = nxt[it];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive_cluster(acc == 0 ? lead_tempty0 : lead_tempty1);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA frees its tensor memory or leaves while the pair still uses it
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)TMEM_COLS));
  }
}

}  // namespace tgcb_gemm
