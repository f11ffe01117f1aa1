// Streaming (one-pass) attention for one head in float32, compiled ahead of time into libtgcb.so.
//
// tgc/analysis/attention.py:97-137 computes softmax(q k^T * scale) v one block of keys at a
// time: scores of the block, the block's row maximum, the running maximum moved to cover it,
// everything accumulated so far rescaled by exp(old max - new max) (0 while the old max is
// -inf), weights exp(score - new max), running sum = sum * correction + block row sum, running
// output = output * correction + weights @ values, and the output divided by the sum at the
// end. The score matrix is never stored.
//
// Widths 64 and 128 run streaming_attention_v (16-byte shared-memory operands, double-buffered
// key/value blocks; below), widths 16 and 32 streaming_attention. In the latter,
// one CTA owns 32 query rows and walks the keys in blocks of 64: the q block stays in
// shared memory, each key/value block is staged once per CTA, the 32 x 64 scores live in
// registers (4 x 4 per thread), row maxima and sums are combined by shuffles across the 16
// threads of a row, and the weights pass through shared memory into the weights @ values
// product. Arithmetic is plain fp32 (no tensor cores), matching tgc's float32 reference up to
// summation order; the key block of 64 is the kernel's, and tgc's `block` argument changes only
// where rounding happens, not the function.
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdint>

#include "internal.h"
#include "tgcb.h"

namespace {

constexpr int BQ = 32;
constexpr int BK = 64;
constexpr int THREADS = 128;

template <int W>
struct Smem {
  static constexpr int QP = W + 1;  // padded rows: consecutive keys/queries fall in different banks
  static constexpr int KP = W + 1;
  static constexpr int PP = BK + 1;
  static constexpr size_t bytes = sizeof(float) * (BQ * QP + BK * KP + BK * W + BQ * PP);
};

template <int W>
__global__ void __launch_bounds__(THREADS) streaming_attention(const float* __restrict__ q, const float* __restrict__ k,
                                                               const float* __restrict__ v, int sq, int sk, float scale,
                                                               float* __restrict__ out) {
  extern __shared__ float smem[];
  using S = Smem<W>;
  float* Qs = smem;
  float* Ks = Qs + BQ * S::QP;
  float* Vs = Ks + BK * S::KP;
  float* Ps = Vs + BK * W;
  constexpr int OC = W / 16;  // output columns per thread

  const int t = threadIdx.x;
  const int ty = t >> 4;  // rows 4*ty .. 4*ty+3
  const int tx = t & 15;  // score columns tx + 16j, output columns tx + 16c
  const long long q0 = (long long)blockIdx.x * BQ;

  for (int i = t; i < BQ * (W / 4); i += THREADS) {
    const int r = i / (W / 4), c4 = i % (W / 4);
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + r < sq) x = __ldg(reinterpret_cast<const float4*>(q + (q0 + r) * W) + c4);
    float* d = Qs + r * S::QP + 4 * c4;
    d[0] = x.x;
    d[1] = x.y;
    d[2] = x.z;
    d[3] = x.w;
  }

  float m[4], l[4], o[4][OC];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int c = 0; c < OC; ++c) o[i][c] = 0.f;
  }

  for (int k0 = 0; k0 < sk; k0 += BK) {
    __syncthreads();  // the previous block's Ks/Vs/Ps are no longer read
    for (int i = t; i < BK * (W / 4); i += THREADS) {
      const int r = i / (W / 4), c4 = i % (W / 4);
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
      if (k0 + r < sk) {
        a = __ldg(reinterpret_cast<const float4*>(k + (long long)(k0 + r) * W) + c4);
        b = __ldg(reinterpret_cast<const float4*>(v + (long long)(k0 + r) * W) + c4);
      }
      float* dk = Ks + r * S::KP + 4 * c4;
      dk[0] = a.x;
      dk[1] = a.y;
      dk[2] = a.z;
      dk[3] = a.w;
      reinterpret_cast<float4*>(Vs + r * W)[c4] = b;
    }
    __syncthreads();

    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 8
    for (int d = 0; d < W; ++d) {
      float qa[4], kb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qa[i] = Qs[(4 * ty + i) * S::QP + d];
#pragma unroll
      for (int j = 0; j < 4; ++j) kb[j] = Ks[(tx + 16 * j) * S::KP + d];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qa[i], kb[j], s[i][j]);
    }

#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float bm = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][j] = (k0 + tx + 16 * j < sk) ? s[i][j] * scale : -INFINITY;
        bm = fmaxf(bm, s[i][j]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, off));
      const float mn = fmaxf(m[i], bm);
      const float corr = (m[i] == -INFINITY) ? 0.f : expf(m[i] - mn);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = expf(s[i][j] - mn);
        Ps[(4 * ty + i) * S::PP + tx + 16 * j] = p;
        rs += p;
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      l[i] = l[i] * corr + rs;
      m[i] = mn;
#pragma unroll
      for (int c = 0; c < OC; ++c) o[i][c] *= corr;
    }
    __syncwarp();  // a row's weights are written and read by the same 16 threads of one warp

    float pv[4][OC];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < OC; ++c) pv[i][c] = 0.f;
#pragma unroll 8
    for (int kk = 0; kk < BK; ++kk) {
      float pa[4], vb[OC];
#pragma unroll
      for (int i = 0; i < 4; ++i) pa[i] = Ps[(4 * ty + i) * S::PP + kk];
#pragma unroll
      for (int c = 0; c < OC; ++c) vb[c] = Vs[kk * W + tx + 16 * c];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < OC; ++c) pv[i][c] = fmaf(pa[i], vb[c], pv[i][c]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < OC; ++c) o[i][c] += pv[i][c];
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const long long r = q0 + 4 * ty + i;
    if (r < sq) {
#pragma unroll
      for (int c = 0; c < OC; ++c) out[r * W + tx + 16 * c] = o[i][c] / l[i];
    }
  }
}

// Widths 64 and 128: the same arithmetic, arranged for the shared-memory pipe. Rows of q, k
// and v sit in shared memory with a padded pitch of W + 4 floats, so every operand read is a
// 16-byte load: a thread's q rows (4 ty + i, shared by the 16 threads of its half-warp, one
// broadcast) and its keys (tx + 16 j, 16 different rows whose 16-byte slots fall on different
// banks) give 64 multiply-adds per 8 loads, and the weights-times-values product reads four
// weights of a row and four value columns (4 tx + 64 c ...) at once. Each key/value block is
// copied with 16-byte cp.async into one of two buffers while the other is in use. The sums run
// in the same order as in streaming_attention: scores over d from 0, the weights@values
// product over the block's keys in order, then added to the running output.
constexpr int PAD = 4;

template <int W>
struct SmemV {
  static constexpr int P = W + PAD;  // q, k, v row pitch (floats)
  static constexpr int PP = BK + PAD;
  static constexpr size_t bytes = sizeof(float) * (BQ * P + 2 * 2 * BK * P + BQ * PP);
};

__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool valid) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}

template <int W>
__global__ void __launch_bounds__(THREADS) streaming_attention_v(const float* __restrict__ q, const float* __restrict__ k,
                                                                 const float* __restrict__ v, int sq, int sk, float scale,
                                                                 float* __restrict__ out) {
  static_assert(W == 64 || W == 128, "the vector kernel covers widths 64 and 128");
  extern __shared__ __align__(16) float vsmem[];
  using S = SmemV<W>;
  constexpr int OV = W / 64;  // float4 output groups per thread: columns 4 tx + 64 c
  float* Qs = vsmem;
  float* KV = Qs + BQ * S::P;  // buffer b: K at KV + 2 b BK P, V right after it
  float* Ps = KV + 2 * 2 * BK * S::P;

  const int t = threadIdx.x;
  const int ty = t >> 4;
  const int tx = t & 15;
  const long long q0 = (long long)blockIdx.x * BQ;
  const int nblk = (sk + BK - 1) / BK;

  for (int i = t; i < BQ * (W / 4); i += THREADS) {
    const int r = i / (W / 4), c4 = i % (W / 4);
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + r < sq) x = __ldg(reinterpret_cast<const float4*>(q + (q0 + r) * W) + c4);
    *reinterpret_cast<float4*>(Qs + r * S::P + 4 * c4) = x;
  }
  auto load_block = [&](int blk) {
    float* Kb = KV + (blk & 1) * 2 * BK * S::P;
    float* Vb = Kb + BK * S::P;
    const int k0 = blk * BK;
    for (int i = t; i < BK * (W / 4); i += THREADS) {
      const int r = i / (W / 4), c4 = i % (W / 4);
      const bool valid = k0 + r < sk;
      const long long src = (long long)(valid ? k0 + r : 0) * W + 4 * c4;
      cp_async16(Kb + r * S::P + 4 * c4, k + src, valid);
      cp_async16(Vb + r * S::P + 4 * c4, v + src, valid);
    }
  };

  float m[4], l[4], o[4][4 * OV];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int c = 0; c < 4 * OV; ++c) o[i][c] = 0.f;
  }

  load_block(0);
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int blk = 0; blk < nblk; ++blk) {
    if (blk + 1 < nblk) load_block(blk + 1);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // this block's copies have landed
    __syncthreads();
    const float* Ks = KV + (blk & 1) * 2 * BK * S::P;
    const float* Vs = Ks + BK * S::P;
    const int k0 = blk * BK;

    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < W; d += 4) {
      float4 qa[4], kb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qa[i] = *reinterpret_cast<const float4*>(Qs + (4 * ty + i) * S::P + d);
#pragma unroll
      for (int j = 0; j < 4; ++j) kb[j] = *reinterpret_cast<const float4*>(Ks + (tx + 16 * j) * S::P + d);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = fmaf(qa[i].x, kb[j].x, s[i][j]);
          s[i][j] = fmaf(qa[i].y, kb[j].y, s[i][j]);
          s[i][j] = fmaf(qa[i].z, kb[j].z, s[i][j]);
          s[i][j] = fmaf(qa[i].w, kb[j].w, s[i][j]);
        }
    }

#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float bm = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][j] = (k0 + tx + 16 * j < sk) ? s[i][j] * scale : -INFINITY;
        bm = fmaxf(bm, s[i][j]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, off));
      const float mn = fmaxf(m[i], bm);
      const float corr = (m[i] == -INFINITY) ? 0.f : expf(m[i] - mn);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = expf(s[i][j] - mn);
        Ps[(4 * ty + i) * S::PP + tx + 16 * j] = p;
        rs += p;
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      l[i] = l[i] * corr + rs;
      m[i] = mn;
#pragma unroll
      for (int c = 0; c < 4 * OV; ++c) o[i][c] *= corr;
    }
    __syncwarp();  // a row's weights are written and read by the same 16 threads of one warp

    float pv[4][4 * OV];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 4 * OV; ++c) pv[i][c] = 0.f;
#pragma unroll 2
    for (int kk = 0; kk < BK; kk += 4) {
      float4 pa[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pa[i] = *reinterpret_cast<const float4*>(Ps + (4 * ty + i) * S::PP + kk);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float4 vb[OV];
#pragma unroll
        for (int c = 0; c < OV; ++c) vb[c] = *reinterpret_cast<const float4*>(Vs + (kk + u) * S::P + 4 * tx + 64 * c);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float p = u == 0 ? pa[i].x : u == 1 ? pa[i].y : u == 2 ? pa[i].z : pa[i].w;
#pragma unroll
          for (int c = 0; c < OV; ++c) {
            pv[i][4 * c + 0] = fmaf(p, vb[c].x, pv[i][4 * c + 0]);
            pv[i][4 * c + 1] = fmaf(p, vb[c].y, pv[i][4 * c + 1]);
            pv[i][4 * c + 2] = fmaf(p, vb[c].z, pv[i][4 * c + 2]);
            pv[i][4 * c + 3] = fmaf(p, vb[c].w, pv[i][4 * c + 3]);
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 4 * OV; ++c) o[i][c] += pv[i][c];
    __syncthreads();  // every thread is done with this buffer before the next prefetch reuses it
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const long long r = q0 + 4 * ty + i;
    if (r < sq) {
#pragma unroll
      for (int c = 0; c < OV; ++c) {
        float4 y;
        y.x = o[i][4 * c + 0] / l[i];
        y.y = o[i][4 * c + 1] / l[i];
        y.z = o[i][4 * c + 2] / l[i];
        y.w = o[i][4 * c + 3] / l[i];
        *reinterpret_cast<float4*>(out + r * W + 4 * tx + 64 * c) = y;
      }
    }
  }
}

template <int W>
int launch_v(const float* q, const float* k, const float* v, int sq, int sk, float* out, cudaStream_t s) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return tgcb_internal_fail(TGCB_E_CUDA, "streaming_attention device", cudaGetErrorString(e));
  static std::atomic<unsigned long long> configured{0};
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    e = cudaFuncSetAttribute(streaming_attention_v<W>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SmemV<W>::bytes);
    if (e != cudaSuccess) return tgcb_internal_fail(TGCB_E_CUDA, "streaming_attention smem", cudaGetErrorString(e));
    configured.fetch_or(bit);
  }
  const float scale = (float)(1.0 / std::sqrt((double)W));
  streaming_attention_v<W><<<(unsigned)((sq + BQ - 1) / BQ), THREADS, SmemV<W>::bytes, s>>>(q, k, v, sq, sk, scale, out);
  e = cudaGetLastError();
  if (e != cudaSuccess) return tgcb_internal_fail(TGCB_E_CUDA, "streaming_attention", cudaGetErrorString(e));
  return TGCB_OK;
}

template <int W>
int launch(const float* q, const float* k, const float* v, int sq, int sk, float* out, cudaStream_t s) {
  // The shared-memory opt-in is a per-device function attribute; setting it again is harmless.
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return tgcb_internal_fail(TGCB_E_CUDA, "streaming_attention device", cudaGetErrorString(e));
  static std::atomic<unsigned long long> configured{0};
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    e = cudaFuncSetAttribute(streaming_attention<W>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Smem<W>::bytes);
    if (e != cudaSuccess) return tgcb_internal_fail(TGCB_E_CUDA, "streaming_attention smem", cudaGetErrorString(e));
    configured.fetch_or(bit);
  }
  const float scale = (float)(1.0 / std::sqrt((double)W));
  streaming_attention<W><<<(unsigned)((sq + BQ - 1) / BQ), THREADS, Smem<W>::bytes, s>>>(q, k, v, sq, sk, scale, out);
  e = cudaGetLastError();
  if (e != cudaSuccess) return tgcb_internal_fail(TGCB_E_CUDA, "streaming_attention", cudaGetErrorString(e));
  return TGCB_OK;
}

}  // namespace

extern "C" int tgcb_streaming_attention_f32(const float* q, const float* k, const float* v, uint32_t sq, uint32_t sk,
                                            uint32_t width, float* out, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
    return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_streaming_attention_f32", "null pointer");
  if (sq == 0 || sk == 0) return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_streaming_attention_f32", "empty sequence");
  if (sq > (1u << 30) || sk > (1u << 30))
    return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_streaming_attention_f32", "sequence longer than 2^30");
  for (const void* p : {(const void*)q, (const void*)k, (const void*)v})
    if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0)
      return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_streaming_attention_f32", "q, k and v must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool out16 = (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  switch (width) {
    case 16: return launch<16>(q, k, v, (int)sq, (int)sk, out, s);
    case 32: return launch<32>(q, k, v, (int)sq, (int)sk, out, s);
    // the vector kernel stores 16-byte groups of the output; an output not 16-byte aligned
    // takes the scalar kernel
    case 64:
      return out16 ? launch_v<64>(q, k, v, (int)sq, (int)sk, out, s) : launch<64>(q, k, v, (int)sq, (int)sk, out, s);
    case 128:
      return out16 ? launch_v<128>(q, k, v, (int)sq, (int)sk, out, s) : launch<128>(q, k, v, (int)sq, (int)sk, out, s);
    default:
      return tgcb_internal_fail(TGCB_E_INVALID, "tgcb_streaming_attention_f32", "width must be 16, 32, 64 or 128");
  }
}
