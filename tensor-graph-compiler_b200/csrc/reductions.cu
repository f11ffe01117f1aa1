// Long reductions and the per-row int8 quantiser, compiled ahead of time into libtgcb.so.
//
// Pairwise sum (tgc/analysis/summation.py:64-85). tgc's _pairwise halves a range at
// size//2 until it holds at most `block` values, sums each block sequentially from 0.0f and
// adds the two halves. With L the deepest level at which every node is still larger than
// `block` plus one, the top L levels are a perfect binary tree over 2^L nodes in index order,
// and every depth-L node needs at most one more split. So:
//   * level 0: thread j computes depth-L node j (a closed form start = j * (n >> L) when 2^L
//     divides n, otherwise a walk of the L halvings), sums it exactly like _pairwise, and
//     256-node groups are combined as perfect trees in shared memory;
//   * levels 1..: the same perfect-tree combine over 256 partials at a time, until one.
//   Where a level is uniform and at least 1024 wide, a block takes 1024 consecutive nodes
//   instead (4 per thread in registers, xor shuffles across lanes, 8 warp partials last):
//   the same perfect tree with one barrier per block instead of eight. When that level has
//   256..16384 blocks, one more block combines all block partials (pairwise_final, a
//   programmatic dependent launch that is resident before the leaves finish).
// Every addition is the one _pairwise performs, so the result is bit-identical.
//
// Sequential sum (summation.py:56-61) is one dependent chain of n float additions; one
// thread runs it with the loads software-pipelined ahead of the chain.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "internal.h"
#include "tgcb.h"

namespace {

int report(int code, const char* what, cudaError_t e) { return tgcb_internal_fail(code, what, cudaGetErrorString(e)); }

constexpr int kGroup = 256;

__device__ __forceinline__ float seq_sum(const float* __restrict__ x, long long start, long long size) {
  float t = 0.0f;
  for (long long i = 0; i < size; ++i) t = __fadd_rn(t, __ldg(x + start + i));
  return t;
}

// Value of the depth-L node [start, start+size) under _pairwise's rules (size <= 2*block+1).
__device__ __forceinline__ float node_value(const float* __restrict__ x, long long start, long long size, int block) {
  if (size <= block) return seq_sum(x, start, size);
  const long long h = size / 2;
  return __fadd_rn(seq_sum(x, start, h), seq_sum(x, start + h, size - h));
}

// Perfect-tree combine of `count` (power of two, <= 256) values held in s[0..count).
__device__ __forceinline__ float tree256(float* s, int count) {
  for (int w = 1; w < count; w *= 2) {
    __syncthreads();
    const int t = threadIdx.x;
    if ((t % (2 * w)) == 0 && t + w < count) s[t] = __fadd_rn(s[t], s[t + w]);
  }
  __syncthreads();
  return s[0];
}

__global__ void __launch_bounds__(kGroup) pairwise_leaves(const float* __restrict__ x, long long n, int L, int block,
                                                          int uniform, float* __restrict__ out) {
  __shared__ float s[kGroup];
  const long long nodes = 1ll << L;
  const long long j = (long long)blockIdx.x * kGroup + threadIdx.x;
  float v = 0.0f;
  if (j < nodes) {
    long long start, size;
    if (uniform) {
      size = n >> L;
      start = j * size;
    } else {
      start = 0;
      size = n;
      for (int lvl = L - 1; lvl >= 0; --lvl) {
        const long long half = size / 2;
        if ((j >> lvl) & 1) {
          start += half;
          size -= half;
        } else {
          size = half;
        }
      }
    }
    if (uniform && size == 8 && block >= 8 && ((reinterpret_cast<uintptr_t>(x + start) & 15u) == 0)) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(x + start));
      const float4 b = __ldg(reinterpret_cast<const float4*>(x + start) + 1);
      float t = 0.0f;
      t = __fadd_rn(t, a.x);
      t = __fadd_rn(t, a.y);
      t = __fadd_rn(t, a.z);
      t = __fadd_rn(t, a.w);
      t = __fadd_rn(t, b.x);
      t = __fadd_rn(t, b.y);
      t = __fadd_rn(t, b.z);
      t = __fadd_rn(t, b.w);
      v = t;
    } else {
      v = node_value(x, start, size, block);
    }
  }
  s[threadIdx.x] = v;
  const int count = (int)(nodes < kGroup ? nodes : kGroup);
  const float r = tree256(s, count);
  if (threadIdx.x == 0) out[blockIdx.x] = r;
}

// Fast path for the perfect part of the tree: each thread takes 4 adjacent values (leaves, or
// partials of a previous level), adds them as ((a+b)+(c+d)), lanes combine by xor shuffles
// 1,2,4,8,16 (adjacent subtrees first), and the 8 warps by a balanced tree in shared memory:
// a perfect tree over 1024 consecutive values per block, the same additions as tree256 makes
// but with one barrier. `count` is a power of two >= 1024.
constexpr int kFastPer = 4;
constexpr int kFastSpan = kGroup * kFastPer;

// Balanced tree over the 8 warp partials of a block; `writer` is the one lane per warp that
// holds its warp's partial. The result is valid on thread 0.
__device__ __forceinline__ float combine_warps(float v, bool writer, float* s) {
  if (writer) s[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.0f;
  if (threadIdx.x == 0) {
    float w[kGroup / 32];
#pragma unroll
    for (int i = 0; i < kGroup / 32; ++i) w[i] = s[i];
#pragma unroll
    for (int width = 1; width < kGroup / 32; width *= 2)
#pragma unroll
      for (int i = 0; i < kGroup / 32; i += 2 * width) w[i] = __fadd_rn(w[i], w[i + width]);
    r = w[0];
  }
  return r;
}

__device__ __forceinline__ float fast_block_tree(float v, float* s) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return combine_warps(v, (threadIdx.x & 31) == 0, s);
}

// 128 leaves of exactly 8 values each (4 KiB from p), read coalesced: in load k the warp reads
// 512 contiguous bytes, lane i the float4 that is half (i & 1) of leaf 16k + i/2. The even
// lane's running sum of its 4 values goes to the odd lane, which finishes the leaf's
// left-to-right chain; xor shuffles 2,4,8,16 build the perfect tree over each load's 16 leaves
// (odd lanes pair with odd lanes), and a register tree over the 8 loads the warp's 128-leaf
// subtree. The result is valid on the odd lanes.
__device__ __forceinline__ float warp_leaves8(const float4* __restrict__ p) {
  const int lane = threadIdx.x & 31;
  float4 q[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) q[k] = __ldg(p + k * 32 + lane);
  float r[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float head = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, q[k].x), q[k].y), q[k].z), q[k].w);
    const float left = __shfl_xor_sync(0xffffffffu, head, 1);
    float t = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(left, q[k].x), q[k].y), q[k].z), q[k].w);
#pragma unroll
    for (int o = 2; o < 32; o <<= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
    r[k] = t;
  }
  return __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                   __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
}

// The 1024 depth-L nodes of this block (uniform leaves), as one perfect-tree value on thread 0.
__device__ __forceinline__ float leaves_block(const float* __restrict__ x, long long n, int L, int block, float* s) {
  const long long size = n >> L;
  if (size == 8 && block >= 8 && ((reinterpret_cast<uintptr_t>(x) & 15u) == 0)) {
    const long long leaf0 = (long long)blockIdx.x * kFastSpan + (threadIdx.x >> 5) * 128;
    const float w = warp_leaves8(reinterpret_cast<const float4*>(x) + leaf0 * 2);
    return combine_warps(w, (threadIdx.x & 31) == 1, s);
  }
  const long long j0 = ((long long)blockIdx.x * kGroup + threadIdx.x) * kFastPer;
  float v[kFastPer];
#pragma unroll
  for (int g = 0; g < kFastPer; ++g) v[g] = node_value(x, (j0 + g) * size, size, block);
  return fast_block_tree(__fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3])), s);
}

__global__ void __launch_bounds__(kGroup) pairwise_leaves_fast(const float* __restrict__ x, long long n, int L,
                                                               int block, float* __restrict__ out) {
  __shared__ float s[kGroup / 32];
  const float r = leaves_block(x, n, L, block, s);
  if (threadIdx.x == 0) out[blockIdx.x] = r;
}

// Perfect tree over C consecutive partials that other blocks of this launch wrote: loads go
// through L2 (ld.global.cg), never the non-coherent read-only path.
template <int C>
__device__ __forceinline__ float chunk_tree(const float* p) {
  float v[C];
#pragma unroll
  for (int i = 0; i < C; ++i) v[i] = __ldcg(p + i);
#pragma unroll
  for (int w = 1; w < C; w *= 2)
#pragma unroll
    for (int i = 0; i < C; i += 2 * w) v[i] = __fadd_rn(v[i], v[i + w]);
  return v[0];
}

// chunk_tree's values for C in 4..32 when the partials are 16-byte aligned. Loading thread t's
// C consecutive partials per thread makes every warp load touch 32 cache lines; instead the
// block loads all 256 * C partials with coalesced 16-byte loads into shared-memory rows of
// C + 1 words (one row per thread: an odd row pitch puts the 32 rows a warp reads on 32
// different banks), then each thread adds its row as the same perfect tree.
constexpr int kStageRow = 33;  // words per staged row: C + 1 for the widest C, 32
template <int C>
__device__ __forceinline__ float staged_chunk_tree(const float* p, float* stage) {
  static_assert(C % 4 == 0 && C <= kStageRow - 1, "a float4 must stay inside one row");
  const float4* p4 = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int k = 0; k < C / 4; ++k) {
    const int j = threadIdx.x + kGroup * k;  // float4 index into the block's 256 * C partials
    const float4 q = __ldcg(p4 + j);
    float* d = stage + (4 * j / C) * (C + 1) + (4 * j) % C;
    d[0] = q.x;
    d[1] = q.y;
    d[2] = q.z;
    d[3] = q.w;
  }
  __syncthreads();
  float v[C];
#pragma unroll
  for (int i = 0; i < C; ++i) v[i] = stage[threadIdx.x * (C + 1) + i];
#pragma unroll
  for (int w = 1; w < C; w *= 2)
#pragma unroll
    for (int i = 0; i < C; i += 2 * w) v[i] = __fadd_rn(v[i], v[i + w]);
  return v[0];
}

// The two launches of a wide uniform sum. The leaf kernel lets its dependent launch start at
// once (programmatic dependent launch), so the final kernel is resident and waiting when the
// last leaf block retires, instead of paying a launch gap. The final kernel (one block) waits
// for the leaf grid's writes, then takes `per` consecutive block partials per thread, adds them
// as a perfect tree, then lanes and warps as before: again the perfect tree over all partials.
__global__ void __launch_bounds__(kGroup) pairwise_leaves_pdl(const float* __restrict__ x, long long n, int L,
                                                              int block, float* __restrict__ out) {
  asm volatile("griddepcontrol.launch_dependents;");
  __shared__ float s[kGroup / 32];
  const float r = leaves_block(x, n, L, block, s);
  if (threadIdx.x == 0) out[blockIdx.x] = r;
}

__global__ void __launch_bounds__(kGroup) pairwise_final(const float* partials, int per, int staged,
                                                          float* __restrict__ out) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float s[kGroup / 32];
  __shared__ float stage[kGroup * kStageRow];
  if (staged) {  // the host sets it only for per in {4, 8, 16, 32} and 16-byte aligned partials
    float v;
    switch (per) {
      case 4: v = staged_chunk_tree<4>(partials, stage); break;
      case 8: v = staged_chunk_tree<8>(partials, stage); break;
      case 16: v = staged_chunk_tree<16>(partials, stage); break;
      default: v = staged_chunk_tree<32>(partials, stage); break;
    }
    const float t = fast_block_tree(v, s);
    if (threadIdx.x == 0) out[0] = t;
    return;
  }
  const float* p = partials + (long long)threadIdx.x * per;
  float v;
  switch (per) {
    case 1: v = chunk_tree<1>(p); break;
    case 2: v = chunk_tree<2>(p); break;
    case 4: v = chunk_tree<4>(p); break;
    case 8: v = chunk_tree<8>(p); break;
    case 16: v = chunk_tree<16>(p); break;
    case 32: v = chunk_tree<32>(p); break;
    default: v = chunk_tree<64>(p); break;
  }
  const float t = fast_block_tree(v, s);
  if (threadIdx.x == 0) out[0] = t;
}

__global__ void __launch_bounds__(kGroup) pairwise_combine_fast(const float* __restrict__ in, float* __restrict__ out) {
  __shared__ float s[kGroup / 32];
  const float4 q = __ldg(reinterpret_cast<const float4*>(in) + (long long)blockIdx.x * kGroup + threadIdx.x);
  const float t4 = __fadd_rn(__fadd_rn(q.x, q.y), __fadd_rn(q.z, q.w));
  const float r = fast_block_tree(t4, s);
  if (threadIdx.x == 0) out[blockIdx.x] = r;
}

__global__ void __launch_bounds__(kGroup) pairwise_combine(const float* __restrict__ in, long long count,
                                                           float* __restrict__ out) {
  __shared__ float s[kGroup];
  const long long j = (long long)blockIdx.x * kGroup + threadIdx.x;
  s[threadIdx.x] = j < count ? in[j] : 0.0f;
  const int c = (int)(count < kGroup ? count : kGroup);
  const float r = tree256(s, c);
  if (threadIdx.x == 0) out[blockIdx.x] = r;
}

__global__ void sequential_chain(const float* __restrict__ x, long long n, float* __restrict__ out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  float t = 0.0f;
  long long i = 0;
  const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
  if (aligned) {
    const float4* v = reinterpret_cast<const float4*>(x);
    const long long nv = n / 4;
    constexpr int D = 16;  // float4 loads kept in flight ahead of the chain
    float4 buf[D];
    long long q = 0;
#pragma unroll
    for (int k = 0; k < D; ++k) buf[k] = (q + k < nv) ? __ldg(v + q + k) : make_float4(0, 0, 0, 0);
    for (; q + D <= nv; q += D) {
#pragma unroll
      for (int k = 0; k < D; ++k) {
        const float4 c = buf[k];
        if (q + D + k < nv) buf[k] = __ldg(v + q + D + k);
        t = __fadd_rn(t, c.x);
        t = __fadd_rn(t, c.y);
        t = __fadd_rn(t, c.z);
        t = __fadd_rn(t, c.w);
      }
    }
    for (long long k = 0; q + k < nv; ++k) {
      const float4 c = buf[k];
      t = __fadd_rn(t, c.x);
      t = __fadd_rn(t, c.y);
      t = __fadd_rn(t, c.z);
      t = __fadd_rn(t, c.w);
    }
    i = nv * 4;
  }
  for (; i < n; ++i) t = __fadd_rn(t, __ldg(x + i));
  *out = t;
}

// The sequential order for long vectors: the chain of n dependent additions runs at the adder's
// latency only if the next values are always at hand, which one thread's own loads cannot
// arrange (a few hundred bytes in flight against the memory latency). So one block of two
// working threads splits the work: thread 32 streams the 16-byte-aligned body of x into a ring
// of shared-memory slots with bulk copies (cp.async.bulk, no multicast), up to
// kSeqSlots * kSeqChunk bytes in flight; thread 0 adds every value from 0.0f in index order,
// reading head, slots and tail in turn, so the additions are exactly summation.sequential's.
// Every wait is bounded; a consumer that gives up writes NaN, and the producer then waits
// (bounded) for its copies in flight before the block exits.
constexpr int kSeqChunk = 8192;   // bytes per slot and per bulk copy
constexpr int kSeqSlots = 16;     // 128 KiB of shared memory
constexpr unsigned kSeqPolls = 1u << 24;
constexpr int kSeqSmem = kSeqSlots * kSeqChunk + 2 * kSeqSlots * 8;

__device__ __forceinline__ bool seq_wait(uint32_t bar, uint32_t parity) {
  for (unsigned i = 0; i < kSeqPolls; ++i) {
    uint32_t ok;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    if (ok) return true;
  }
  return false;
}

__global__ void __launch_bounds__(64) sequential_staged(const float* __restrict__ x, long long n, float* __restrict__ out) {
  extern __shared__ __align__(128) unsigned char seq_smem[];
  __shared__ volatile int abort_flag;
  __shared__ volatile long long consumed;
  unsigned long long* bars = reinterpret_cast<unsigned long long*>(seq_smem + kSeqSlots * kSeqChunk);
  const uint32_t ring = static_cast<uint32_t>(__cvta_generic_to_shared(seq_smem));
  const uint32_t bar0 = static_cast<uint32_t>(__cvta_generic_to_shared(bars));  // full[s], then empty[s]
  const uintptr_t addr = reinterpret_cast<uintptr_t>(x);
  long long head = (long long)(((16u - (addr & 15u)) & 15u) / 4u);  // floats before the first 16-byte boundary
  if (head > n) head = n;
  const long long body = ((n - head) / 4) * 4;  // whole 16-byte units
  const long long body_bytes = body * 4;
  const long long chunks = (body_bytes + kSeqChunk - 1) / kSeqChunk;
  if (threadIdx.x == 0) {
    for (int q = 0; q < 2 * kSeqSlots; ++q)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8u * q));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_flag = 0;
    consumed = 0;
  }
  __syncthreads();
  if (threadIdx.x == 32) {
    long long issued = 0;
    for (long long c = 0; c < chunks; ++c) {
      const int slot = (int)(c % kSeqSlots);
      const long long round = c / kSeqSlots;
      if (round > 0 && !seq_wait(bar0 + 8u * (kSeqSlots + slot), (uint32_t)((round - 1) & 1))) break;
      if (abort_flag) break;
      const long long off = c * kSeqChunk;
      const uint32_t bytes = (uint32_t)(body_bytes - off < kSeqChunk ? body_bytes - off : kSeqChunk);
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar0 + 8u * slot), "r"(bytes) : "memory");
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       ring + slot * kSeqChunk),
                   "l"(reinterpret_cast<const char*>(x + head) + off), "r"(bytes), "r"(bar0 + 8u * slot)
                   : "memory");
      issued = c + 1;
    }
    if (abort_flag) {
      // the consumer gave up: let the copies still in flight land before the block exits
      for (long long c = consumed; c < issued; ++c)
        seq_wait(bar0 + 8u * (int)(c % kSeqSlots), (uint32_t)((c / kSeqSlots) & 1));
    }
  } else if (threadIdx.x == 0) {
    float t = 0.0f;
    for (long long i = 0; i < head; ++i) t = __fadd_rn(t, __ldg(x + i));
    for (long long c = 0; c < chunks; ++c) {
      const int slot = (int)(c % kSeqSlots);
      if (!seq_wait(bar0 + 8u * slot, (uint32_t)((c / kSeqSlots) & 1))) {
        abort_flag = 1;
        *out = __int_as_float(0x7fc00000);
        return;
      }
      const long long off = c * kSeqChunk;
      const int nv = (int)((body_bytes - off < kSeqChunk ? body_bytes - off : kSeqChunk) / 16);
      const float4* p = reinterpret_cast<const float4*>(seq_smem + slot * kSeqChunk);
      int q = 0;
      for (; q + 8 <= nv; q += 8) {
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = p[q + j];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          t = __fadd_rn(t, v[j].x);
          t = __fadd_rn(t, v[j].y);
          t = __fadd_rn(t, v[j].z);
          t = __fadd_rn(t, v[j].w);
        }
      }
      for (; q < nv; ++q) {
        const float4 v = p[q];
        t = __fadd_rn(t, v.x);
        t = __fadd_rn(t, v.y);
        t = __fadd_rn(t, v.z);
        t = __fadd_rn(t, v.w);
      }
      consumed = c + 1;
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar0 + 8u * (kSeqSlots + slot)) : "memory");
    }
    for (long long i = head + body; i < n; ++i) t = __fadd_rn(t, __ldg(x + i));
    *out = t;
  }
}

// One CTA per row. The row stays in registers between the max pass and the quantise pass.
template <int PER_THREAD>
__global__ void __launch_bounds__(256) quantise_rows(const float* __restrict__ x, long long rows, long long cols,
                                                     int8_t* __restrict__ q, float* __restrict__ scale) {
  __shared__ float red[8];
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* row = x + r * cols;
    float v[PER_THREAD];
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < PER_THREAD; ++k) {
      const long long c = threadIdx.x + (long long)k * 256;
      v[k] = c < cols ? __ldg(row + c) : 0.0f;
      const float a = fabsf(v[k]);
      m = (a > m || a != a) ? a : m;
    }
    for (long long c = threadIdx.x + (long long)PER_THREAD * 256; c < cols; c += 256) {
      const float a = fabsf(__ldg(row + c));
      m = (a > m || a != a) ? a : m;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float other = __shfl_xor_sync(0xffffffffu, m, o);
      m = (other > m || other != other) ? other : m;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    float mm = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) mm = (red[w] > mm || red[w] != red[w]) ? red[w] : mm;
    __syncthreads();
    // scale = largest / 127 computed in double and read back as float32; 1.0 for a zero row.
    const float s = (mm == 0.0f) ? 1.0f : (float)((double)mm / 127.0);
    if (threadIdx.x == 0) scale[r] = s;
    int8_t* qrow = q + r * cols;
#pragma unroll
    for (int k = 0; k < PER_THREAD; ++k) {
      const long long c = threadIdx.x + (long long)k * 256;
      if (c < cols) {
        float t = rintf(__fdiv_rn(v[k], s));
        t = fminf(fmaxf(t, -128.0f), 127.0f);
        qrow[c] = (int8_t)(int)t;
      }
    }
    for (long long c = threadIdx.x + (long long)PER_THREAD * 256; c < cols; c += 256) {
      float t = rintf(__fdiv_rn(__ldg(row + c), s));
      t = fminf(fmaxf(t, -128.0f), 127.0f);
      qrow[c] = (int8_t)(int)t;
    }
  }
}

// Rows whose length is a multiple of 1024 (and 16-byte aligned): one CTA per row, each thread
// holding V float4 of its row in registers (columns 4(t + 256k) .. +3). max|x| is exact in any
// order and the quantisation is elementwise, so this layout changes no result; it only makes
// every load 16 bytes and every store 4 bytes wide.
//
// max|x| is the unsigned maximum of the sign-cleared bit patterns: for non-negative floats the
// unsigned order is the numeric order and every NaN pattern lies above +inf, so a NaN anywhere
// in the row gives a NaN maximum (and every element of that row takes the exact quotient).
//
// rint(x / s) without a division per element: t = x * (1/s) with the correctly rounded
// reciprocal differs from the correctly rounded quotient by at most 2 * 2^-24 * |x/s| (two
// roundings), below 1.6e-5 for |x/s| <= 128 (|x| <= m here). Unless t lies within 3e-5 of a
// half-integer, both round to the same integer; near a half-integer the exact quotient
// decides. t - rint(t) is exact for |t| <= 128 (Sterbenz). When m and 1/s are finite (uniform
// over the row) every |x / s| is at most 127 * (1 + 2^-21) even for a subnormal s, so the
// rounded value lies in [-127, 127] and needs no clamp; rows with a non-finite m or 1/s take
// the exact quotient with the clamp to [-128, 127] for every element.
template <int V>
__global__ void __launch_bounds__(256) quantise_rows_vec(const float* __restrict__ x, long long cols,
                                                          int8_t* __restrict__ q, float* __restrict__ scale) {
  __shared__ unsigned red[8];
  const long long r = blockIdx.x;
  const float4* row = reinterpret_cast<const float4*>(x + r * cols);
  float4 v[V];
#pragma unroll
  for (int k = 0; k < V; ++k) v[k] = __ldg(row + threadIdx.x + 256 * k);
  unsigned m = 0u;
#pragma unroll
  for (int k = 0; k < V; ++k) {
    m = max(m, __float_as_uint(v[k].x) & 0x7fffffffu);
    m = max(m, __float_as_uint(v[k].y) & 0x7fffffffu);
    m = max(m, __float_as_uint(v[k].z) & 0x7fffffffu);
    m = max(m, __float_as_uint(v[k].w) & 0x7fffffffu);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  unsigned mb = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) mb = max(mb, red[w]);
  const float mm = __uint_as_float(mb);
  const float s = (mm == 0.0f) ? 1.0f : (float)((double)mm / 127.0);
  if (threadIdx.x == 0) scale[r] = s;
  const float inv = __fdiv_rn(1.0f, s);
  char4* qrow = reinterpret_cast<char4*>(q + r * cols);
  if (isfinite(inv) && isfinite(mm)) {
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float e[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
      signed char b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float t = e[i] * inv;
        float qi = rintf(t);
        if (fabsf(0.5f - fabsf(t - qi)) <= 3e-5f) qi = rintf(__fdiv_rn(e[i], s));
        b[i] = (signed char)(int)qi;
      }
      qrow[threadIdx.x + 256 * k] = make_char4(b[0], b[1], b[2], b[3]);
    }
  } else {
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float e[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
      signed char b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float qi = rintf(__fdiv_rn(e[i], s));
        b[i] = (signed char)(int)fminf(fmaxf(qi, -128.0f), 127.0f);
      }
      qrow[threadIdx.x + 256 * k] = make_char4(b[0], b[1], b[2], b[3]);
    }
  }
}

int levels_for(uint64_t n, int block) {
  // deepest L with floor(n / 2^(L-1)) > block, i.e. every node above depth L is internal
  int L = 0;
  while ((n >> L) > (uint64_t)block) ++L;
  return L;
}

}  // namespace

extern "C" {

size_t tgcb_sum_pairwise_scratch_bytes(uint64_t n, int block) {
  if (n == 0 || block < 1) return 0;
  const int L = levels_for(n, block);
  uint64_t count = 1ull << L;
  size_t total = 0;
  while (true) {
    const uint64_t groups = (count + kGroup - 1) / kGroup;
    total += groups * sizeof(float);
    if (groups <= 1) break;
    count = groups;
  }
  return (total + 255) & ~size_t(255);
}

int tgcb_sum_pairwise_f32(const float* x, uint64_t n, int block, float* out, void* scratch, size_t scratch_bytes,
                          void* stream) {
  if (x == nullptr || out == nullptr) return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_sum_pairwise_f32", "null pointer");
  if (n == 0) return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_sum_pairwise_f32", "there is nothing to sum");
  if (block < 1) return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_sum_pairwise_f32", "a block must hold at least one value");
  const size_t need = tgcb_sum_pairwise_scratch_bytes(n, block);
  if (scratch == nullptr || scratch_bytes < need)
    return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_sum_pairwise_f32", "scratch is smaller than tgcb_sum_pairwise_scratch_bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int L = levels_for(n, block);
  const long long nodes = 1ll << L;
  const int uniform = (n % (uint64_t)nodes) == 0 ? 1 : 0;
  float* buf = static_cast<float*>(scratch);
  // Two launches where the leaf level fills 256..16384 blocks of 1024 nodes: the leaf partials,
  // then one block that combines them, launched as a programmatic dependent of the first.
  if (uniform && nodes >= 256ll * kFastSpan && nodes <= 16384ll * kFastSpan) {
    const long long grid = nodes / kFastSpan;
    pairwise_leaves_pdl<<<(unsigned)grid, kGroup, 0, s>>>(x, (long long)n, L, block, buf);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return report(TGCB_E_CUDA, "pairwise_leaves_pdl", e);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kGroup);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const int per = (int)(grid / kGroup);
    const int staged = per >= 4 && per <= 32 && (reinterpret_cast<uintptr_t>(buf) & 15u) == 0;
    e = cudaLaunchKernelEx(&cfg, pairwise_final, (const float*)buf, per, staged, out);
    if (e != cudaSuccess) return report(TGCB_E_CUDA, "pairwise_final", e);
    return TGCB_OK;
  }
  // Perfect-tree levels of 1024 values per block where the level is wide enough; the
  // 256-per-block kernels finish narrow levels and irregular (non-uniform) leaves.
  const bool fast0 = uniform && nodes >= kFastSpan;
  long long groups = fast0 ? nodes / kFastSpan : (nodes + kGroup - 1) / kGroup;
  float* dst = groups == 1 ? out : buf;
  if (fast0)
    pairwise_leaves_fast<<<(unsigned)groups, kGroup, 0, s>>>(x, (long long)n, L, block, dst);
  else
    pairwise_leaves<<<(unsigned)groups, kGroup, 0, s>>>(x, (long long)n, L, block, uniform, dst);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return report(TGCB_E_CUDA, "pairwise_leaves", e);
  float* src = buf;
  float* next = buf + groups;
  while (groups > 1) {
    const bool fast = groups >= kFastSpan && groups % kFastSpan == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
    const long long g2 = fast ? groups / kFastSpan : (groups + kGroup - 1) / kGroup;
    float* d = g2 == 1 ? out : next;
    if (fast)
      pairwise_combine_fast<<<(unsigned)g2, kGroup, 0, s>>>(src, d);
    else
      pairwise_combine<<<(unsigned)g2, kGroup, 0, s>>>(src, groups, d);
    e = cudaGetLastError();
    if (e != cudaSuccess) return report(TGCB_E_CUDA, "pairwise_combine", e);
    src = next;
    next = next + g2;
    groups = g2;
  }
  return TGCB_OK;
}

int tgcb_sum_perfect_tree_f32(const float* partials, uint32_t count, float* out, void* stream) {
  if (partials == nullptr || out == nullptr)
    return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_sum_perfect_tree_f32", "null pointer");
  if (count == 0 || count > (uint32_t)kGroup || (count & (count - 1)) != 0)
    return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_sum_perfect_tree_f32", "count must be a power of two from 1 to 256");
  pairwise_combine<<<1, kGroup, 0, static_cast<cudaStream_t>(stream)>>>(partials, (long long)count, out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return report(TGCB_E_CUDA, "pairwise_combine", e);
  return TGCB_OK;
}

int tgcb_sum_sequential_f32(const float* x, uint64_t n, float* out, void* stream) {
  if (x == nullptr || out == nullptr) return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_sum_sequential_f32", "null pointer");
  if (n == 0) return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_sum_sequential_f32", "there is nothing to sum");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n < (1u << 16)) {
    sequential_chain<<<1, 32, 0, s>>>(x, (long long)n, out);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return report(TGCB_E_CUDA, "sequential_chain", e);
    return TGCB_OK;
  }
  cudaError_t e = cudaFuncSetAttribute(sequential_staged, cudaFuncAttributeMaxDynamicSharedMemorySize, kSeqSmem);
  if (e != cudaSuccess) return report(TGCB_E_CUDA, "sequential_staged shared memory", e);
  sequential_staged<<<1, 64, kSeqSmem, s>>>(x, (long long)n, out);
  e = cudaGetLastError();
  if (e != cudaSuccess) return report(TGCB_E_CUDA, "sequential_staged", e);
  return TGCB_OK;
}

int tgcb_quantise_rows_i8(const float* x, int64_t rows, int64_t cols, int8_t* q, float* scale, void* stream) {
  if (x == nullptr || q == nullptr || scale == nullptr)
    return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_quantise_rows_i8", "null pointer");
  if (rows < 1 || cols < 1) return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_quantise_rows_i8", "there is nothing to quantise");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(q)) & 15u) == 0;
  const long long per = cols / 1024;  // float4 per thread in quantise_rows_vec
  if (aligned && cols % 1024 == 0 && rows <= 0x7fffffffll && (per == 1 || per == 2 || per == 4 || per == 8 || per == 16)) {
    if (per == 1) quantise_rows_vec<1><<<(unsigned)rows, 256, 0, s>>>(x, cols, q, scale);
    if (per == 2) quantise_rows_vec<2><<<(unsigned)rows, 256, 0, s>>>(x, cols, q, scale);
    if (per == 4) quantise_rows_vec<4><<<(unsigned)rows, 256, 0, s>>>(x, cols, q, scale);
    if (per == 8) quantise_rows_vec<8><<<(unsigned)rows, 256, 0, s>>>(x, cols, q, scale);
    if (per == 16) quantise_rows_vec<16><<<(unsigned)rows, 256, 0, s>>>(x, cols, q, scale);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return report(TGCB_E_CUDA, "quantise_rows_vec", e);
    return TGCB_OK;
  }
  const unsigned grid = (unsigned)(rows < 148 * 8 ? rows : 148 * 8);
  if (cols <= 256 * 4)
    quantise_rows<4><<<grid, 256, 0, s>>>(x, rows, cols, q, scale);
  else
    quantise_rows<16><<<grid, 256, 0, s>>>(x, rows, cols, q, scale);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return report(TGCB_E_CUDA, "quantise_rows", e);
  return TGCB_OK;
}

}  // extern "C"

// ----------------------------------------------------------------------------- no-alloc variant
//
// For callers that cannot allocate device memory (see include/tgcb.h): the pairwise sum's
// partials live in this file-scope device array instead of caller scratch. On the host its
// name is only a stand-in for the symbol, never a device address; the address is looked up per
// device with cudaGetSymbolAddress (by tgcb_init, or by the first call on a device tgcb_init has
// not set up) and then passed to the unchanged entry point.
static __device__ __align__(256) unsigned char g_noalloc_pairwise_scratch[TGCB_NOALLOC_SCRATCH_BYTES];

namespace {
void* g_noalloc_scratch_ptr[kTgcbMaxDevices] = {};
std::mutex g_noalloc_mutex;

int noalloc_lookup_locked(int device) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_pairwise_scratch);
  if (e != cudaSuccess) return report(TGCB_E_CUDA, "cudaGetSymbolAddress of the built-in scratch array", e);
  g_noalloc_scratch_ptr[device] = p;
  return TGCB_OK;
}
}  // namespace

int tgcb_internal_noalloc_setup(int device) {
  if (device < 0 || device >= kTgcbMaxDevices)
    return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_init", "device index out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  return noalloc_lookup_locked(device);
}

extern "C" int tgcb_sum_pairwise_f32_noalloc(const float* x, uint64_t n, int block, float* out, void* stream) {
  if (x == nullptr || out == nullptr)
    return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_sum_pairwise_f32_noalloc", "null pointer");
  if (n == 0) return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_sum_pairwise_f32_noalloc", "there is nothing to sum");
  if (block < 1)
    return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_sum_pairwise_f32_noalloc", "a block must hold at least one value");
  const size_t need = tgcb_sum_pairwise_scratch_bytes(n, block);
  if (need > TGCB_NOALLOC_SCRATCH_BYTES)
    return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_sum_pairwise_f32_noalloc",
                              "this length needs more scratch than the built-in 1 MiB array (at most 9 * 2^25 - 1 "
                              "values at block 8); use tgcb_sum_pairwise_f32 with caller scratch");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return report(TGCB_E_CUDA, "cudaGetDevice", e);
  if (dev < 0 || dev >= kTgcbMaxDevices)
    return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_sum_pairwise_f32_noalloc", "device index out of range");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_scratch_ptr[dev] == nullptr) {
      const int rc = noalloc_lookup_locked(dev);  // tgcb_init never ran for this device
      if (rc != TGCB_OK) return rc;
    }
    scratch = g_noalloc_scratch_ptr[dev];
  }
  return tgcb_sum_pairwise_f32(x, n, block, out, scratch, TGCB_NOALLOC_SCRATCH_BYTES, stream);
}
