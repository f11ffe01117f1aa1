// Persistent tcgen05 GEMM for sm_100a: D[M,N] = A[M,K] @ B[K,N] with a generated epilogue.
//
// One CTA per SM loops over 128x256 output tiles. Warp 0 is the TMA producer, warp 1 issues
// tcgen05.mma from one thread, warps 2..17 are the epilogue. Operands are staged through a
// 4-deep ring of shared-memory stages, each 128 bytes of K per row (32 tf32 or 128 int8
// values) in the 128-byte swizzled layout that TMA writes and the UMMA descriptors read.
// The accumulator lives in tensor memory: two 256-column fp32/int32 buffers, so the
// epilogue drains tile t while the tensor core fills tile t+1.
//
// K-major and MN-major operands are both native (tcgen05 accepts MN-major TF32 and INT8),
// so a transposed operand costs nothing: the graph's transpose nodes become descriptor bits.
// No TMA load here uses cluster multicast.
//
// Every wait on an mbarrier is bounded by a wall-clock budget; a CTA that exceeds it sets a
// shared abort flag, records a status code in args.status and unwinds (all roles watch the
// flag), and the TMEM it holds is freed before it exits.
#pragma once
#include "jit_common.cuh"

struct __align__(64) TgcbTmaDesc {
  unsigned long long raw[16];
};

namespace tgcb_gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int STAGES = 4;
constexpr int ROW_BYTES = 128;
constexpr int A_STAGE = BM * ROW_BYTES;   // 16 KB
constexpr int B_STAGE = BN * ROW_BYTES;   // 32 KB
constexpr int EPI_WARPS = 16;  // four per TMEM lane quadrant, 64 columns each
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int TMEM_COLS = 2 * BN;
constexpr int BAR_BYTES = 256;
// Each epilogue warp transposes 32 rows x 8 columns at a time through shared memory.
constexpr int STAGE_WORDS = 32 * 8;
constexpr int EPI_STAGE_BYTES = EPI_WARPS * STAGE_WORDS * 4;
constexpr int SMEM_BYTES = STAGES * (A_STAGE + B_STAGE) + BAR_BYTES + EPI_STAGE_BYTES + 1024;
constexpr unsigned long long WAIT_BUDGET_NS = 4000000000ull;  // 4 s

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  uint32_t r;
  asm volatile("{ .reg .u64 t; cvta.to.shared.u64 t, %1; cvt.u32.u64 %0, t; }" : "=r"(r) : "l"(p));
  return r;
}

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void bar_arrive_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: true when the phase completed, false when this CTA is aborting.
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status, int code) {
  unsigned long long start = 0;
  for (uint32_t it = 0;; ++it) {
    if (bar_try(bar, parity)) return true;
    if ((it & 255u) == 255u) {
      if (*abort_flag) return false;
      const unsigned long long t = now_ns();
      if (start == 0) {
        start = t;
      } else if (t - start > WAIT_BUDGET_NS) {
        *abort_flag = 1;
        tgcb_fail(status, code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const TgcbTmaDesc* desc, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<unsigned long long>(desc)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// The same through a 3-D view (x within a 32-column chunk, y = row, z = chunk): one copy of
// several 32-column chunks, which the 2-D form needs one 4 KB copy each for.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const TgcbTmaDesc* desc, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<unsigned long long>(desc)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

// Whether an MN-major operand is loaded through the 3-D view (the runtime encodes that view for
// the same operands: tgcb_operand_desc.chunks > 0). tf32 MN-major stages are 32-column chunks of
// 4 KB; tiled copies that small fill shared memory at well under half the rate of 16 KB ones,
// so a whole stage of chunks is one copy when the MN extent is a multiple of 32. int8 MN-major
// stages are 16 KB boxes already.
// TGCB_CHUNKED_MN (set by the generated source, default 1) turns the 3-D form off for
// comparisons.
#ifndef TGCB_CHUNKED_MN
#define TGCB_CHUNKED_MN 1
#endif
__host__ __device__ constexpr bool chunked_mn(bool int8, bool mn_major, int mn_extent) {
  return TGCB_CHUNKED_MN && !int8 && mn_major && mn_extent % 32 == 0;
}

// Shared-memory matrix descriptor with sm_100 version bits. layout 2 = 128-byte swizzle in
// 16-byte units (8-row atoms); layout 1 = 128-byte swizzle in 32-byte units (4-row atoms),
// the only layout tcgen05 accepts for MN-major 32-bit (tf32) operands.
__device__ __forceinline__ unsigned long long umma_desc(uint32_t start, uint32_t lbo, uint32_t sbo, uint32_t layout = 2) {
  unsigned long long d = 0;
  d |= (unsigned long long)((start >> 4) & 0x3FFFu);
  d |= (unsigned long long)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (unsigned long long)((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  d |= (unsigned long long)(layout & 7u) << 61;
  return d;
}

template <bool INT8>
__device__ __forceinline__ void mma(uint32_t d_tmem, unsigned long long a, unsigned long long b, uint32_t idesc, uint32_t accumulate) {
  if constexpr (INT8) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p; }" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
  } else {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p; }" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
  }
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int M, int N, int K, bool INT8, bool A_MN, bool B_MN, class Epi>
__device__ __forceinline__ void gemm_body(const TgcbArgs& args, const TgcbTmaDesc* ta, const TgcbTmaDesc* tb) {
  constexpr int EB = INT8 ? 1 : 4;              // element bytes
  constexpr int KB = ROW_BYTES / EB;            // K elements per stage
  constexpr int MMA_K = 32 / EB;                // K elements per tcgen05.mma (32 bytes)
  constexpr int KSTEPS = KB / MMA_K;            // 4
  constexpr int NUM_KB = (K + KB - 1) / KB;
  constexpr int TILES_M = (M + BM - 1) / BM;
  constexpr int TILES_N = (N + BN - 1) / BN;
  constexpr int NUM_TILES = TILES_M * TILES_N;
  constexpr uint32_t STAGE_TX = A_STAGE + B_STAGE;
  // MN-major tf32 tiles are written by TMA with SWIZZLE_128B_ATOM_32B (layout 1, 4-row atoms);
  // MN-major int8 tiles use the ordinary 128-byte swizzle (layout 2, 8-row atoms).
  constexpr uint32_t MN_LAYOUT = INT8 ? 2u : 1u;
  constexpr uint32_t MN_SBO = INT8 ? 1024u : 512u;
  // Instruction descriptor: D format, A/B formats, majors, N>>3, M>>4.
  constexpr uint32_t IDESC = (INT8 ? (2u << 4) : (1u << 4)) | (INT8 ? (1u << 7) : (2u << 7)) |
                             (INT8 ? (1u << 10) : (2u << 10)) | ((A_MN ? 1u : 0u) << 15) | ((B_MN ? 1u : 0u) << 16) |
                             ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

  extern __shared__ unsigned char tgcb_smem_raw[];
  const uint32_t raw = smem_addr(tgcb_smem_raw);
  unsigned char* smem = tgcb_smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  const uint32_t sA = smem_addr(smem);
  const uint32_t sB = sA + STAGES * A_STAGE;
  unsigned long long* bars = reinterpret_cast<unsigned long long*>(smem + STAGES * (A_STAGE + B_STAGE));
  const uint32_t bar0 = smem_addr(bars);
  // full[s] = bar0 + 8*s, empty[s] = bar0 + 8*(STAGES+s), tfull[a], tempty[a] after those.
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (blockDim.x != THREADS) {
    if (threadIdx.x == 0) tgcb_fail(args.status, TGCB_STATUS_BAD_LAUNCH);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      bar_init(full_bar(s), 1);
      bar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      bar_init(tfull_bar(a), 1);
      bar_init(tempty_bar(a), EPI_WARPS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"((uint32_t)TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(ta)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(tb)) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < NUM_TILES; tile += gridDim.x) {
        const int tm = tile / TILES_N;  // N fastest: CTAs running together share A panels in L2
        const int tn = tile % TILES_N;
        for (int kb = 0; kb < NUM_KB; ++kb) {
          if (!bar_wait(empty_bar(stage), phase ^ 1u, abort_flag, args.status, TGCB_STATUS_TIMEOUT_PRODUCER)) goto producer_done;
          bar_arrive_expect(full_bar(stage), STAGE_TX);
          const uint32_t a_dst = sA + stage * A_STAGE;
          const uint32_t b_dst = sB + stage * B_STAGE;
          if (!A_MN) {
            tma_load_2d(a_dst, ta, kb * KB, tm * BM, full_bar(stage));
          } else if constexpr (chunked_mn(INT8, A_MN, M)) {
            tma_load_3d(a_dst, ta, 0, kb * KB, tm * BM / 32, full_bar(stage));
          } else {
#pragma unroll
            for (int c = 0; c < BM * EB / ROW_BYTES; ++c)
              tma_load_2d(a_dst + c * (KB * ROW_BYTES), ta, tm * BM + c * (ROW_BYTES / EB), kb * KB, full_bar(stage));
          }
          if (!B_MN) {
            tma_load_2d(b_dst, tb, kb * KB, tn * BN, full_bar(stage));
          } else if constexpr (chunked_mn(INT8, B_MN, N)) {
            tma_load_3d(b_dst, tb, 0, kb * KB, tn * BN / 32, full_bar(stage));
          } else {
#pragma unroll
            for (int c = 0; c < BN * EB / ROW_BYTES; ++c)
              tma_load_2d(b_dst + c * (KB * ROW_BYTES), tb, tn * BN + c * (ROW_BYTES / EB), kb * KB, full_bar(stage));
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = blockIdx.x; tile < NUM_TILES; tile += gridDim.x) {
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
          const uint32_t a_base = sA + stage * A_STAGE;
          const uint32_t b_base = sB + stage * B_STAGE;
#pragma unroll
          for (int k = 0; k < KSTEPS; ++k) {
            // K-major: advance 32 bytes inside the swizzled 128-byte row; SBO = 8 rows.
            // MN-major: advance MMA_K rows of 128 bytes; LBO = distance between 128-byte MN
            // chunks; SBO = one swizzle atom of K rows (8 rows, or 4 for the tf32 32-byte layout).
            const unsigned long long adesc = A_MN ? umma_desc(a_base + k * MMA_K * ROW_BYTES, KB * ROW_BYTES, MN_SBO, MN_LAYOUT)
                                                  : umma_desc(a_base + k * 32, 16, 1024);
            const unsigned long long bdesc = B_MN ? umma_desc(b_base + k * MMA_K * ROW_BYTES, KB * ROW_BYTES, MN_SBO, MN_LAYOUT)
                                                  : umma_desc(b_base + k * 32, 16, 1024);
            mma<INT8>(d, adesc, bdesc, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit(empty_bar(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(tfull_bar(acc));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    const int ew = warp - 2;
    const int quad = warp & 3;         // TMEM lanes 32*quad .. 32*quad+31 (the warp's rows)
    const int part = ew >> 2;          // which quarter of the 256 columns this warp drains
    uint32_t* stage = reinterpret_cast<uint32_t*>(smem + STAGES * (A_STAGE + B_STAGE) + BAR_BYTES) + ew * STAGE_WORDS;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < NUM_TILES; tile += gridDim.x) {
      const int tm = tile / TILES_N;
      const int tn = tile % TILES_N;
      const long long row0 = (long long)tm * BM + quad * 32;
      if constexpr (Epi::VEC4) {
        // 8 columns of the warp's 32 rows per step: lane = row coming out of TMEM; after the
        // transpose lane takes 4 consecutive columns (one 16-byte access) of row 16*it + lane/2.
        // 16-byte slots are XOR-swizzled by (row/4)%2 so the writes (8 rows per phase) and the
        // reads (4 rows x 2 slots per phase) each hit all 32 banks once.
        constexpr int C8 = BN / 4 / 8;
        const int cbase = part * (BN / 4);
        uint4* st4 = reinterpret_cast<uint4*>(stage);
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
        if (lane == 0) bar_arrive(tempty_bar(acc));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
        continue;
      }
      constexpr int CHUNKS = BN / 32;  // 8-column chunks per warp: 64 columns each
      const int chunk0 = part * CHUNKS;
      // Side inputs of the first chunk are fetched before waiting for the accumulator,
      // so their latency overlaps the tensor-core work of this tile.
      typename Epi::Loads cur[8], nxt[8];
#pragma unroll
      for (int it = 0; it < 8; ++it)
        cur[it] = Epi::load(args, row0 + 4 * it + (lane >> 3), (long long)tn * BN + chunk0 * 8 + (lane & 7));
      bool ok = true;
      if (lane == 0) ok = bar_wait(tfull_bar(acc), acc_phase, abort_flag, args.status, TGCB_STATUS_TIMEOUT_EPILOGUE);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      tc_fence_after();
#pragma unroll 1
      for (int chunk = chunk0; chunk < chunk0 + CHUNKS; ++chunk) {
        uint32_t r[8];
        tmem_ld8(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN + chunk * 8), r);
        // lane = row on the way in; on the way out each lane takes one column of one of four
        // rows, so side-input loads and stores run along rows (32-byte segments). The 8-word
        // rows are XOR-swizzled by row/4 so both the writes and the reads are conflict-free.
#pragma unroll
        for (int j = 0; j < 8; ++j) stage[lane * 8 + (j ^ (lane >> 2))] = r[j];
        __syncwarp();
        const long long col0 = (long long)tn * BN + chunk * 8;
        if (chunk + 1 < chunk0 + CHUNKS) {
#pragma unroll
          for (int it = 0; it < 8; ++it) nxt[it] = Epi::load(args, row0 + 4 * it + (lane >> 3), col0 + 8 + (lane & 7));
        }
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int rr = 4 * it + (lane >> 3);
          const int cc = lane & 7;
          const uint32_t bits = stage[rr * 8 + (cc ^ it)];
          if constexpr (INT8) {
            Epi::apply(args, row0 + rr, col0 + cc, (int)bits, cur[it]);
          } else {
            Epi::apply(args, row0 + rr, col0 + cc, __uint_as_float(bits), cur[it]);
          }
        }
        __syncwarp();
#pragma unroll
        for (int it = 0; it < 8; ++it) cur[it] = nxt[it];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(tempty_bar(acc));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)TMEM_COLS));
  }
}

}  // namespace tgcb_gemm
