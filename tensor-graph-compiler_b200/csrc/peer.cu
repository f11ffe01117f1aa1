// Peer memory over NVLink and the gradient all-reduce that runs on it.
//
// tgc models data parallelism in one process and prices the gradient all-reduce with a ring
// model (tgc/parallel/collective.py:76-113); it never moves bytes between devices. Here each
// rank is a process driving one GPU. The ranks of one box share device memory through CUDA IPC
// (cudaIpcGetMemHandle / cudaIpcOpenMemHandle: plain peer mappings over NVLink/NVSwitch, no
// multicast objects), and tgcb_peer_allreduce_avg_f32 averages gradients that lie at the same
// offsets of every rank's arena in place, in two shots by one kernel per rank:
//
//   1. every rank announces that its values are final (a release store into a flag word of
//      every rank) and waits until all ranks have;
//   2. rank r owns share r of the 16-byte vectors of the segments; for each vector of its share
//      it loads the values of ranks 0, 1, ..., world-1 (its own from local memory, the others
//      over NVLink), adds them in that order, divides by world, and stores the result into
//      every rank's arena;
//   3. every CTA counts itself finished on its own rank once its stores are fenced; the last
//      one tells every rank that this rank is done (release, system scope); CTA 0 waits until
//      every rank has, so the kernel ends only when this rank's segments hold the averages.
//
// Each element is summed once, by its owner, in rank order, and the same bits are stored on
// every rank: the result is the same on all ranks and on every run. Flags are monotonic per
// slot (epoch e: ready and done words hold e, the finished count reaches e x CTAs), so nothing is reset between
// calls; calls in different slots may run at the same time. Every wait is bounded (4 s of
// %globaltimer): a rank that gives up records TGCB_STATUS_TIMEOUT_PEER in the device status
// word and returns, and the host reads it with tgcb_status.
#include <cuda_runtime.h>

#include <cstring>

#include "internal.h"
#include "tgcb.h"

namespace {

constexpr int kMaxPeers = TGCB_MAX_PEERS;
constexpr int kSlots = TGCB_PEER_SLOTS;
constexpr int kMaxSegments = TGCB_PEER_MAX_SEGMENTS;
constexpr int kThreads = 512;
constexpr unsigned long long kWaitBudgetNs = 4000000000ull;
constexpr int kStatusTimeoutPeer = 5;  // device status code (the kernels' TGCB_STATUS_* family)

struct PeerParams {
  float4* base[kMaxPeers];     // every rank's arena base (this rank's: its local address)
  unsigned* flags[kMaxPeers];  // every rank's flag words
  unsigned long long seg_off[kMaxSegments];  // first 16-byte vector of each segment (from the base)
  unsigned long long seg_end[kMaxSegments];  // vectors in segments 0 .. s
  int nseg, rank, world, slot;
  unsigned epoch;
  int* status;
};

// flag words of one rank: ready[slot][src], done[slot][src], then finished[slot] (this rank's
// CTAs that have finished storing, counted locally)
__device__ __forceinline__ unsigned* ready_word(unsigned* flags, int slot, int src) { return flags + slot * kMaxPeers + src; }
__device__ __forceinline__ unsigned* done_word(unsigned* flags, int slot, int src) {
  return flags + kSlots * kMaxPeers + slot * kMaxPeers + src;
}
__device__ __forceinline__ unsigned* finished_word(unsigned* flags, int slot) { return flags + 2 * kSlots * kMaxPeers + slot; }

__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ float4 ld_volatile4(const float4* p) {
  float4 v;
  asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

// Wait until *p has reached `target` (modulo 2^32, within 2^31); false when the budget runs out
// (recording the timeout) or another thread has recorded a failure.
__device__ bool wait_reached(const unsigned* p, unsigned target, int* status) {
  unsigned long long start = 0;
  for (unsigned it = 0;; ++it) {
    if ((int)(ld_acquire_sys(p) - target) >= 0) return true;
    if (*reinterpret_cast<volatile int*>(status) != 0) return false;
    __nanosleep(64);
    if ((it & 255u) == 255u) {
      const unsigned long long t = globaltimer();
      if (start == 0) {
        start = t;
      } else if (t - start > kWaitBudgetNs) {
        atomicCAS(status, 0, kStatusTimeoutPeer);
        return false;
      }
    }
  }
}

__device__ __forceinline__ unsigned long long vector_address(const PeerParams& p, unsigned long long i) {
  unsigned long long first = 0;
  for (int s = 0; s < p.nseg; ++s) {
    if (i < p.seg_end[s]) return p.seg_off[s] + (i - first);
    first = p.seg_end[s];
  }
  return 0;  // not reached: i < seg_end[nseg - 1]
}

// U vectors per thread at a time, their WORLD x U loads issued before any addition, so that
// about eight 16-byte loads per thread are in flight whatever the number of ranks (remote
// loads are latency-bound over NVLink).
template <int WORLD, int U>
__device__ __forceinline__ void reduce_vectors(const PeerParams& p, const unsigned long long (&e)[U], int n) {
  float4 v[U][WORLD];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (u < n) {
#pragma unroll
      for (int r = 0; r < WORLD; ++r) v[u][r] = r == p.rank ? p.base[r][e[u]] : ld_volatile4(p.base[r] + e[u]);
    }
  }
  const float w = (float)WORLD;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (u < n) {
      float4 acc = v[u][0];
#pragma unroll
      for (int r = 1; r < WORLD; ++r) {
        acc.x = __fadd_rn(acc.x, v[u][r].x);
        acc.y = __fadd_rn(acc.y, v[u][r].y);
        acc.z = __fadd_rn(acc.z, v[u][r].z);
        acc.w = __fadd_rn(acc.w, v[u][r].w);
      }
      acc = make_float4(__fdiv_rn(acc.x, w), __fdiv_rn(acc.y, w), __fdiv_rn(acc.z, w), __fdiv_rn(acc.w, w));
#pragma unroll
      for (int r = 0; r < WORLD; ++r) p.base[r][e[u]] = acc;
    }
  }
}

template <int WORLD>
__device__ void reduce_share(const PeerParams& p) {
  constexpr int U = WORLD >= 8 ? 2 : 8 / WORLD;  // 8 ranks: 16 loads in flight, 121 us against 130 for one
  const unsigned long long total = p.seg_end[p.nseg - 1];
  const unsigned long long share = (total + WORLD - 1) / WORLD;
  const unsigned long long lo = (unsigned long long)p.rank * share;
  const unsigned long long hi = lo + share < total ? lo + share : total;
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long i = lo + (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < hi; i += U * stride) {
    unsigned long long e[U];
    int n = 0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const unsigned long long k = i + u * stride;
      e[u] = k < hi ? vector_address(p, k) : 0;
      n += k < hi ? 1 : 0;
    }
    reduce_vectors<WORLD, U>(p, e, n);
  }
}

__global__ void __launch_bounds__(kThreads) allreduce_avg(const PeerParams p) {
  unsigned* own = p.flags[p.rank];
  // 1. this rank's values are final; wait until every rank's are. Every CTA announces it (the
  // same value, so the stores are idempotent): no CTA waits on one that may not be resident.
  if (threadIdx.x < p.world) st_release_sys(ready_word(p.flags[threadIdx.x], p.slot, p.rank), p.epoch);
  int ok = 1;
  if (threadIdx.x < p.world) ok = wait_reached(ready_word(own, p.slot, threadIdx.x), p.epoch, p.status) ? 1 : 0;
  if (!__syncthreads_and(ok)) return;
  // 2. this rank's share, summed in rank order and stored on every rank
  switch (p.world) {
    case 1: reduce_share<1>(p); break;
    case 2: reduce_share<2>(p); break;
    case 3: reduce_share<3>(p); break;
    case 4: reduce_share<4>(p); break;
    case 5: reduce_share<5>(p); break;
    case 6: reduce_share<6>(p); break;
    case 7: reduce_share<7>(p); break;
    default: reduce_share<8>(p); break;
  }
  // 3. this CTA's stores are visible system-wide; it counts itself finished on this rank, and
  // the last of this rank's CTAs tells every rank that this rank is done (one store per rank)
  __threadfence_system();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0)
    last = (int)(atom_add_acq_rel_gpu(finished_word(own, p.slot), 1u) + 1u - p.epoch * gridDim.x) == 0 ? 1 : 0;
  __syncthreads();
  if (last && threadIdx.x < p.world) st_release_sys(done_word(p.flags[threadIdx.x], p.slot, p.rank), p.epoch);
  if (blockIdx.x != 0) return;
  // CTA 0 ends only when every rank has finished storing into this rank's arena
  if (threadIdx.x < p.world) wait_reached(done_word(own, p.slot, threadIdx.x), p.epoch, p.status);
}

}  // namespace

extern "C" {

int tgcb_peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr || bytes == 0)
    return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_peer_alloc", "null output or zero size");
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return tgcb_internal_fail(TGCB_E_CUDA, "tgcb_peer_alloc: cudaMalloc", cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return tgcb_internal_fail(TGCB_E_CUDA, "tgcb_peer_alloc: exporting the buffer", cudaGetErrorString(e));
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return TGCB_OK;
}

int tgcb_peer_free(void* ptr) {
  if (ptr == nullptr) return TGCB_OK;
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return tgcb_internal_fail(TGCB_E_CUDA, "tgcb_peer_free", cudaGetErrorString(e));
  return TGCB_OK;
}

int tgcb_peer_open(const void* handle, void** ptr) {
  if (handle == nullptr || ptr == nullptr) return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_peer_open", "null argument");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return tgcb_internal_fail(TGCB_E_CUDA, "tgcb_peer_open", cudaGetErrorString(e));
  return TGCB_OK;
}

int tgcb_peer_close(void* ptr) {
  if (ptr == nullptr) return TGCB_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return tgcb_internal_fail(TGCB_E_CUDA, "tgcb_peer_close", cudaGetErrorString(e));
  return TGCB_OK;
}

int tgcb_peer_allreduce_avg_f32(const tgcb_peer_group* g, const tgcb_segment* segs, int n_segs, int slot, uint32_t epoch,
                                int ctas, void* stream) {
  if (g == nullptr || segs == nullptr) return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_peer_allreduce_avg_f32", "null argument");
  if (g->world < 1 || g->world > kMaxPeers || g->rank < 0 || g->rank >= g->world)
    return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_peer_allreduce_avg_f32", "rank or world out of range (world 1..8)");
  if (n_segs < 1 || n_segs > kMaxSegments)
    return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_peer_allreduce_avg_f32", "1..8 segments");
  if (slot < 0 || slot >= kSlots) return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_peer_allreduce_avg_f32", "slot out of range (0..3)");
  if (epoch == 0) return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_peer_allreduce_avg_f32", "epochs start at 1");
  if (ctas < 1 || ctas > 1024) return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_peer_allreduce_avg_f32", "1..1024 CTAs");
  PeerParams p;
  std::memset(&p, 0, sizeof(p));
  for (int r = 0; r < g->world; ++r) {
    if (g->bases[r] == nullptr || g->flags[r] == nullptr ||
        (reinterpret_cast<uintptr_t>(g->bases[r]) & 15u) != 0 || (reinterpret_cast<uintptr_t>(g->flags[r]) & 3u) != 0)
      return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_peer_allreduce_avg_f32", "every rank needs a 16-byte aligned base and flags");
    p.base[r] = static_cast<float4*>(g->bases[r]);
    p.flags[r] = g->flags[r];
  }
  unsigned long long end = 0;
  for (int s = 0; s < n_segs; ++s) {
    if (segs[s].offset % 16 != 0 || segs[s].count % 4 != 0 || segs[s].count == 0)
      return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_peer_allreduce_avg_f32",
                                "segments start on 16 bytes and hold a positive multiple of 4 floats");
    if (segs[s].offset > g->bytes || segs[s].count > (g->bytes - segs[s].offset) / 4)
      return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_peer_allreduce_avg_f32", "a segment reaches past the peer buffers");
    p.seg_off[s] = segs[s].offset / 16;
    end += segs[s].count / 4;
    p.seg_end[s] = end;
  }
  p.nseg = n_segs;
  p.rank = g->rank;
  p.world = g->world;
  p.slot = slot;
  p.epoch = epoch;
  int rc = tgcb_internal_status_word(&p.status);
  if (rc != TGCB_OK) return rc;
  allreduce_avg<<<ctas, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return tgcb_internal_fail(TGCB_E_CUDA, "tgcb_peer_allreduce_avg_f32: launch", cudaGetErrorString(e));
  return TGCB_OK;
}

}  // extern "C"
