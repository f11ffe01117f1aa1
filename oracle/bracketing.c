/*
 * CPU restatements of float32 summation orders. TEST INFRASTRUCTURE ONLY.
 * Built with -O2 -ffp-contract=off and no fast-math so every addition is one IEEE float add.
 *
 * tgc's orders (tgc/analysis/summation.py):
 *   oracle_sequential   :56-61   one accumulator from 0.0f, left to right
 *   oracle_pairwise     :64-85   halve at size//2 until <= block, blocks summed sequentially
 *   oracle_partitioned  :115-131 parts with edges round(k*n/parts), partials summed sequentially
 *
 * The declared bracketings of the backend's reduction kernels (tgcb/codegen.py, jit_common.cuh):
 *   oracle_row_tree     row kernels: T threads, thread t sums columns t, t+T, ... sequentially
 *                       from 0; 32 lanes combined as a balanced tree in lane order; T/32 warp
 *                       partials combined as a balanced tree in warp order. op 0 = sum, 1 = max.
 *   oracle_col_parts    column kernels: P row blocks of L rows summed sequentially per column,
 *                       then the P partials sequentially.
 *   oracle_full_chunks  full reductions: G chunks of `chunk` elements, each reduced like one
 *                       row of T=256 threads; then the G partials reduced like one row.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

static float add(float a, float b) {
  volatile float r = a + b; /* keep the rounding to float explicit */
  return r;
}

static float nanmax(float a, float b) { return (a != a || a > b) ? a : b; }

float oracle_sequential(const float* x, int64_t n) {
  float t = 0.0f;
  for (int64_t i = 0; i < n; ++i) t = add(t, x[i]);
  return t;
}

static float pairwise_rec(const float* x, int64_t n, int block) {
  if (n <= block) return oracle_sequential(x, n);
  int64_t mid = n / 2;
  float l = pairwise_rec(x, mid, block);
  float r = pairwise_rec(x + mid, n - mid, block);
  return add(l, r);
}

float oracle_pairwise(const float* x, int64_t n, int block) { return pairwise_rec(x, n, block); }

float oracle_partitioned(const float* x, int64_t n, int64_t parts) {
  float* partial = (float*)malloc(sizeof(float) * (size_t)parts);
  for (int64_t k = 0; k < parts; ++k) {
    /* Python's round(k * n / parts): round half to even of the exact quotient */
    double q0 = (double)k * (double)n / (double)parts;
    double q1 = (double)(k + 1) * (double)n / (double)parts;
    int64_t e0 = (int64_t)nearbyint(q0), e1 = (int64_t)nearbyint(q1);
    partial[k] = oracle_sequential(x + e0, e1 - e0);
  }
  float t = oracle_sequential(partial, parts);
  free(partial);
  return t;
}

static float tree(float* v, int count, int op) {
  for (int w = 1; w < count; w *= 2)
    for (int i = 0; i + w < count; i += 2 * w) v[i] = op ? nanmax(v[i], v[i + w]) : add(v[i], v[i + w]);
  return v[0];
}

/* One row of `cols` values reduced by T threads (T a multiple of 32, power of two). */
static float row_tree_one(const float* row, int64_t cols, int T, int op) {
  float lanes[1024];
  float warps[32];
  for (int t = 0; t < T; ++t) {
    float acc = op ? -INFINITY : 0.0f;
    for (int64_t c = t; c < cols; c += T) acc = op ? nanmax(acc, row[c]) : add(acc, row[c]);
    lanes[t] = acc;
  }
  int W = T / 32;
  for (int w = 0; w < W; ++w) warps[w] = tree(lanes + 32 * w, 32, op);
  return tree(warps, W, op);
}

void oracle_row_tree(const float* x, int64_t rows, int64_t cols, int T, int op, float* out) {
  for (int64_t r = 0; r < rows; ++r) out[r] = row_tree_one(x + r * cols, cols, T, op);
}

void oracle_col_parts(const float* x, int64_t rows, int64_t cols, int64_t L, int op, float* out) {
  int64_t P = (rows + L - 1) / L;
  float* part = (float*)malloc(sizeof(float) * (size_t)P);
  for (int64_t c = 0; c < cols; ++c) {
    for (int64_t p = 0; p < P; ++p) {
      float acc = op ? -INFINITY : 0.0f;
      int64_t r1 = (p + 1) * L < rows ? (p + 1) * L : rows;
      for (int64_t r = p * L; r < r1; ++r) acc = op ? nanmax(acc, x[r * cols + c]) : add(acc, x[r * cols + c]);
      part[p] = acc;
    }
    float acc = op ? -INFINITY : 0.0f;
    for (int64_t p = 0; p < P; ++p) acc = op ? nanmax(acc, part[p]) : add(acc, part[p]);
    out[c] = acc;
  }
  free(part);
}

float oracle_full_chunks(const float* x, int64_t n, int64_t chunk, int op) {
  int64_t G = (n + chunk - 1) / chunk;
  float* part = (float*)malloc(sizeof(float) * (size_t)G);
  for (int64_t g = 0; g < G; ++g) {
    int64_t e0 = g * chunk;
    int64_t len = (e0 + chunk < n ? chunk : n - e0);
    part[g] = row_tree_one(x + e0, len, 256, op);
  }
  float r = row_tree_one(part, G, 256, op);
  free(part);
  return r;
}
