// Shared device code for the kernels tgcb generates at compile time (NVRTC, sm_100a).
//
// Every generated kernel takes one TgcbArgs by value: the arena base (one device
// allocation holding every materialised value at the offsets the planner chose), the
// graph inputs (read-only, never copied when the caller's device buffer is usable as is)
// and a device status word where a kernel that had to give up records why.
//
// The block reductions here fix the bracketing every row/full reduction uses, so that a
// CPU restatement (oracle/bracketing.c) reproduces the result bit for bit:
//   1. thread t of a W-warp block holds a partial it summed sequentially;
//   2. the 32 lanes of a warp combine by xor shuffles with offsets 1, 2, 4, 8, 16, which is
//      a balanced binary tree over lanes in order (lane i with lane i^1 first);
//   3. the W warp partials are combined as a balanced binary tree in warp order
//      (W is a power of two), computed redundantly by every thread from shared memory.
#pragma once

#ifdef __CUDACC_RTC__
typedef unsigned int uint32_t;
typedef unsigned long long uint64_t;
typedef signed char int8_t;
typedef long long int64_t;
#else
#include <cstdint>
#endif

#define TGCB_MAX_INPUTS 48

struct TgcbArgs {
  char* arena;
  const char* in[TGCB_MAX_INPUTS];
  int* status;
};

// Status codes a kernel may write into args.status (first writer wins).
#define TGCB_STATUS_OK 0
#define TGCB_STATUS_TIMEOUT_PRODUCER 1
#define TGCB_STATUS_TIMEOUT_MMA 2
#define TGCB_STATUS_TIMEOUT_EPILOGUE 3
#define TGCB_STATUS_BAD_LAUNCH 4

#ifndef INFINITY
#define INFINITY __int_as_float(0x7f800000)
#endif

// Approximate functions for TF32 GEMM epilogues only, whose results are compared at TF32
// tolerance; every other kernel calls CUDA's accurate functions. tanh is the hardware's own
// (PTX tanh.approx.f32: one special-function instruction, maximum relative error about 2^-11,
// the size of one TF32 rounding of an input), and sigmoid(u) = 0.5 + 0.5 tanh(u / 2) takes the
// same instruction. On the MLP block's GELU epilogue the first GEMM runs 6% faster with it than
// with tanh built from the hardware exponential and reciprocal (two such instructions and more
// arithmetic per element, in warps that share issue slots with the MMA and TMA warps), and the
// block's largest error against the oracle is unchanged (TF32 rounding of the operands
// dominates).
__device__ __forceinline__ float tgcb_tanh_approx(float u) {
  float r;
  asm("tanh.approx.f32 %0, %1;" : "=f"(r) : "f"(u));
  return r;
}
__device__ __forceinline__ float tgcb_sigmoid_approx(float u) { return 0.5f + 0.5f * tgcb_tanh_approx(0.5f * u); }

__device__ __forceinline__ long long tgcb_min_ll(long long a, long long b) { return a < b ? a : b; }
__device__ __forceinline__ long long tgcb_max_ll(long long a, long long b) { return a > b ? a : b; }

__device__ __forceinline__ void tgcb_fail(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

template <typename T>
__device__ __forceinline__ T tgcb_nanmax(T a, T b) {
  // torch.amax / maximum propagate NaN; a NaN accumulator stays NaN, a NaN operand wins.
  return (a != a || a > b) ? a : b;
}

template <typename T>
__device__ __forceinline__ T tgcb_shfl_xor(T v, int offset) {
  return __shfl_xor_sync(0xffffffffu, v, offset);
}

template <typename T, int W>
__device__ __forceinline__ T tgcb_tree_combine_sum(const T* p) {
  // balanced tree over W values in order; W in {1, 2, 4, 8, 16, 32}
  T v[W];
#pragma unroll
  for (int i = 0; i < W; ++i) v[i] = p[i];
#pragma unroll
  for (int width = 1; width < W; width *= 2) {
#pragma unroll
    for (int i = 0; i < W; i += 2 * width) v[i] = v[i] + v[i + width];
  }
  return v[0];
}

template <typename T, int W>
__device__ __forceinline__ T tgcb_tree_combine_max(const T* p) {
  T v[W];
#pragma unroll
  for (int i = 0; i < W; ++i) v[i] = p[i];
#pragma unroll
  for (int width = 1; width < W; width *= 2) {
#pragma unroll
    for (int i = 0; i < W; i += 2 * width) v[i] = tgcb_nanmax(v[i], v[i + width]);
  }
  return v[0];
}

// Reductions over one row handled by the W warps of a row group (W = threads per row / 32).
// `tid` is the thread's index within its row group; `smem` holds W slots for this group.
// Every thread of the CTA must call these the same number of times (the row groups of a
// CTA run in lockstep), since W > 1 uses __syncthreads.
template <typename T, int W>
__device__ __forceinline__ T tgcb_group_sum(T v, T* smem, int tid) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) v = v + tgcb_shfl_xor(v, o);
  if (W == 1) return v;
  if ((tid & 31) == 0) smem[tid >> 5] = v;
  __syncthreads();
  T r = tgcb_tree_combine_sum<T, W>(smem);
  __syncthreads();
  return r;
}

template <typename T, int W>
__device__ __forceinline__ T tgcb_group_max(T v, T* smem, int tid) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) v = tgcb_nanmax(v, tgcb_shfl_xor(v, o));
  if (W == 1) return v;
  if ((tid & 31) == 0) smem[tid >> 5] = v;
  __syncthreads();
  T r = tgcb_tree_combine_max<T, W>(smem);
  __syncthreads();
  return r;
}

template <typename T, int W>
__device__ __forceinline__ T tgcb_block_sum(T v, T* smem) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) v = v + tgcb_shfl_xor(v, o);
  if (W == 1) return v;
  if ((threadIdx.x & 31) == 0) smem[threadIdx.x >> 5] = v;
  __syncthreads();
  T r = tgcb_tree_combine_sum<T, W>(smem);
  __syncthreads();
  return r;
}

template <typename T, int W>
__device__ __forceinline__ T tgcb_block_max(T v, T* smem) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) v = tgcb_nanmax(v, tgcb_shfl_xor(v, o));
  if (W == 1) return v;
  if ((threadIdx.x & 31) == 0) smem[threadIdx.x >> 5] = v;
  __syncthreads();
  T r = tgcb_tree_combine_max<T, W>(smem);
  __syncthreads();
  return r;
}
