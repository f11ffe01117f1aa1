/*
 * tgcb: B200 (sm_100a) execution backend for tgc's compiled graphs. C-ABI of libtgcb.so.
 *
 * tgc runs a compiled graph as generated Python calling torch against one arena
 * (tgc/runtime/executor.py:91-122, tgc/codegen/emit.py:165-209). This library is the seam
 * that replaces the last two steps of compile_graph (emit + exec) and the call
 * CompiledGraph.function(arena, inputs) (executor.py:52-88):
 *
 *   tgc step                                   | entry point here
 *   -------------------------------------------+------------------------------------------
 *   emit() writes source              emit.py:165 | host side writes CUDA source per plan
 *   compile(source) + exec     executor.py:110-113 | tgcb_compile_cubin + tgcb_module_load
 *   namespace["compiled"]         executor.py:113 | tgcb_plan_create
 *   compiled(arena, inputs)        executor.py:79 | tgcb_plan_run
 *
 * plus the reduction and quantisation kernels tgc keeps outside the graph:
 *   summation.sequential / pairwise (tgc/analysis/summation.py:56-85)
 *                                           -> tgcb_sum_sequential_f32 / tgcb_sum_pairwise_f32
 *   quantize.symmetric_scheme + quantise per row (tgc/analysis/quantize.py:90-128, 229-240)
 *                                           -> tgcb_quantise_rows_i8
 *
 * Conventions: every function returns 0 on success or a negative TGCB_E_* status and never
 * traps; tgcb_last_error() returns the calling thread's message for the last failure.
 * Pointers are device pointers unless named host_*. Streams are cudaStream_t passed as
 * void* (NULL = the legacy default stream). No torch types cross this boundary.
 */
#ifndef TGCB_H_
#define TGCB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TGCB_OK 0
#define TGCB_E_INVALID (-1)  /* bad argument: maps to ConfigError / AllocationError */
#define TGCB_E_CUDA (-2)     /* CUDA runtime failure */
#define TGCB_E_COMPILE (-3)  /* NVRTC rejected the generated source: maps to CodegenError */
#define TGCB_E_DEVICE (-4)   /* a kernel reported a device-side timeout in the status word */
#define TGCB_E_NOT_FOUND (-5)

#define TGCB_MAX_INPUTS 48

typedef struct tgcb_module tgcb_module;
typedef struct tgcb_plan tgcb_plan;

/* Where a GEMM operand lives and how TMA tiles it (row-major storage rows x cols). */
typedef struct tgcb_operand_desc {
  int32_t input_index;   /* >= 0: graph input slot; -1: arena */
  uint32_t elem_bytes;   /* 4 (float32 read as tf32) or 1 (int8) */
  uint64_t arena_offset; /* bytes from the arena base when input_index < 0 */
  uint64_t rows;
  uint64_t cols;
  uint32_t box_cols;     /* TMA box extent along the contiguous axis (elements) */
  uint32_t box_rows;     /* TMA box extent along rows */
  uint32_t swizzle;      /* 0: 128-byte swizzle of 16-byte units; 1: of 32-byte units (tf32 MN-major) */
  uint32_t chunks;       /* 0: a 2-D map of boxes box_cols x box_rows. c > 0 (swizzle 1, cols a multiple
                            of 32): a 3-D view (32 columns, rows, cols / 32 chunks) whose box takes c
                            chunks of 32 columns x box_rows rows at once, laid out chunk after chunk:
                            one copy of box_rows x 32c values instead of c copies of 4 KB */
} tgcb_operand_desc;

/* One kernel launch of a plan. Plain kernels take TgcbArgs; GEMM kernels take TgcbArgs
 * and two tensor maps that tgcb_plan_run encodes from a and b; a chain (is_gemm 3: two GEMMs
 * in one launch of clusters of two CTAs, the second reading the first one's output rows) takes
 * four, from a, b, a2 and b2. For any GEMM launch with counter_bytes > 0 (a chain's per-row-
 * block counters, a K-split GEMM's per-region counters) tgcb_plan_run zeroes that many bytes of
 * arena at counter_offset before every launch. Every pair of a chain must be resident at once:
 * the first launch checks the device's cluster occupancy and fails with TGCB_E_INVALID when it
 * cannot hold them. */
typedef struct tgcb_launch_desc {
  char kernel[96];
  uint32_t grid[3];
  uint32_t block[3];
  uint32_t smem_bytes;
  uint32_t is_gemm;      /* 0: plain kernel; 1: GEMM; 2: GEMM launched as clusters of two CTAs; 3: chain */
  tgcb_operand_desc a;
  tgcb_operand_desc b;
  tgcb_operand_desc a2;  /* is_gemm 3 only */
  tgcb_operand_desc b2;  /* is_gemm 3 only */
  uint64_t counter_offset; /* GEMM launches: bytes from the arena base, 4-byte aligned */
  uint64_t counter_bytes;  /* 0: no counters (required > 0 for is_gemm 3) */
} tgcb_launch_desc;

/* Library version string, naming the NVRTC version that compiles generated kernels in this
 * process (the first libnvrtc.so.12 the process loaded). */
const char* tgcb_version(void);

/* Message of the calling thread's last failure ("" if none). */
const char* tgcb_last_error(void);

/* Select `device` (0 .. 15), allocate its status word, resolve the driver's tensor-map encoder
 * and look up the device address of tgcb_sum_pairwise_f32_noalloc's built-in scratch array.
 * Idempotent per device; each call repeats the look-up. Replaces nothing in tgc (tgc is
 * single-device CPU). */
int tgcb_init(int device);

/* Number of CUDA devices visible (0 on a host without a GPU). Never fails. */
int tgcb_device_count(void);

/* Compile CUDA C++ source for sm_100a with NVRTC (-std=c++17 --fmad=false, include_dir on
 * the include path). On success *cubin is malloc'd (free with tgcb_free); on a compile
 * error *log holds NVRTC's log (malloc'd) and TGCB_E_COMPILE is returned.
 * Replaces: compile(module.source, "<tgc>", "exec") (tgc/runtime/executor.py:112). */
int tgcb_compile_cubin(const char* source, const char* include_dir, const char* const* extra_options,
                       int n_extra_options, void** cubin, size_t* cubin_size, char** log);

void tgcb_free(void* p);

/* Load a cubin produced by tgcb_compile_cubin into the current context. */
int tgcb_module_load(const void* cubin, size_t size, tgcb_module** out);
/* Releases the module once the launches its plans queued have finished: every tgcb_plan_run*
 * records an event behind its launches, per device and stream, and this call waits for those
 * events only (other work on the devices keeps running). Destroy the module's plans first.
 * Returns TGCB_E_CUDA, and keeps the module loaded, when a wait fails (its kernels may still be
 * running); a plan run captured into a CUDA graph records its event as a graph node, so the
 * wait covers the graph's last replay. */
int tgcb_module_unload(tgcb_module* m);

/* Resolve each launch's kernel in `m` and keep the descriptors.
 * Replaces: namespace["compiled"] (tgc/runtime/executor.py:113). */
int tgcb_plan_create(tgcb_module* m, const tgcb_launch_desc* launches, int n_launches, uint64_t arena_bytes,
                     tgcb_plan** out);
void tgcb_plan_destroy(tgcb_plan* p);

/* Declare that the plan's kernels read graph inputs 0 .. n_inputs-1 (the generated code indexes
 * them without checks). Every later run of the plan then refuses, with TGCB_E_INVALID and
 * before queueing anything, an input table shorter than n_inputs or one holding a null pointer
 * among them, instead of letting a kernel read through it. A plan whose count was never set
 * (0) checks nothing. The C-side counterpart of the refusal of a call that lacks a feed in
 * CompiledGraph.__call__ (tgc/runtime/executor.py:74-78). */
int tgcb_plan_set_input_count(tgcb_plan* p, int n_inputs);

/* Launch every kernel of the plan in order on `stream`. `arena` is a device allocation of at
 * least arena_bytes (256-byte aligned); inputs[i] is the device address of graph input i
 * (read only). Asynchronous: returns after the launches are queued.
 * Replaces: compiled(arena, inputs) (tgc/runtime/executor.py:79, generated by emit.py:165-209). */
int tgcb_plan_run(tgcb_plan* p, void* arena, const void* const* inputs, int n_inputs, void* stream);

/* Number of launches a plan queues per run. */
int tgcb_plan_launch_count(const tgcb_plan* p);

/* tgcb_plan_run restricted to launches [first, first + count). Running the ranges of a plan
 * back to back on one stream is the same as tgcb_plan_run; a data-parallel step splits its
 * plan where a gradient becomes final and starts that gradient's all-reduce on another
 * stream while the remaining launches run (tgc/parallel/collective.py:339-379 models this
 * overlap; here it is executed). */
int tgcb_plan_run_range(tgcb_plan* p, int first, int count, void* arena, const void* const* inputs, int n_inputs,
                        void* stream);

/* tgcb_plan_run with a CUDA event recorded on `stream` before the first launch and after
 * every launch; waits for the stream and writes each launch's device time in milliseconds to
 * ms[0 .. launch_count). The measurement tgc's runtime/profile.py:91-145 takes with
 * perf_counter around the whole call, taken per kernel on the device instead. */
int tgcb_plan_run_profiled(tgcb_plan* p, void* arena, const void* const* inputs, int n_inputs, void* stream,
                           float* ms);

/* Queue a kernel on `stream` that spins for about `ns` nanoseconds (capped at 10 ms) and
 * exits. Benchmarks put it before a timed region so the launches behind it start back to
 * back instead of waiting on the host. */
int tgcb_delay(uint64_t ns, void* stream);

/* Read (and with clear != 0, reset) the device status word of the current device.
 * Synchronises the device. *status = 0 means every kernel so far completed normally. */
int tgcb_status(int clear, int* status);

/* Pairwise sum, block 8, bit-exact to tgc/analysis/summation.py:64-85 (_pairwise): halve the
 * range at size//2 until it is <= block, sum blocks sequentially from 0.0f, add halves.
 * `scratch` must hold tgcb_sum_pairwise_scratch_bytes(n, block) bytes. Writes *out (device). */
size_t tgcb_sum_pairwise_scratch_bytes(uint64_t n, int block);
int tgcb_sum_pairwise_f32(const float* x, uint64_t n, int block, float* out, void* scratch, size_t scratch_bytes,
                          void* stream);

/* The top levels of a pairwise sum split across GPUs: a perfect binary tree over `count`
 * partials in index order (count a power of two, 1..256): ((p0+p1)+(p2+p3))+... . When each
 * of 2^k GPUs holds one depth-k node of tgc's _pairwise halving (tgc/analysis/summation.py:
 * 77-85) and has summed it with tgcb_sum_pairwise_f32, the gathered partials combined here give
 * the whole vector's _pairwise value bit for bit. Writes *out (device). */
int tgcb_sum_perfect_tree_f32(const float* partials, uint32_t count, float* out, void* stream);

/* One head of attention in one pass over the keys, float32, replacing
 * tgc/analysis/attention.py:97-137 (streaming_attention): out = softmax(q k^T / sqrt(width)) v
 * with the running maximum and sum rescaled per block of keys, the score matrix never stored.
 * q [sq, width], k and v [sk, width], out [sq, width], all row-major float32 device arrays,
 * 16-byte aligned; width 16, 32, 64 or 128. Agrees with tgc's float32 result up to summation
 * order (the kernel's key block is 64). */
int tgcb_streaming_attention_f32(const float* q, const float* k, const float* v, uint32_t sq, uint32_t sk,
                                 uint32_t width, float* out, void* stream);

/* Sequential sum from 0.0f left to right, bit-exact to tgc/analysis/summation.py:56-61. */
int tgcb_sum_sequential_f32(const float* x, uint64_t n, float* out, void* stream);

/* No counterpart in the reference: tgc runs on the CPU and never needs device memory.
 *
 * The pairwise sum above, for callers that cannot allocate device memory themselves: code
 * running inside a host callback or a memory-pool-restricted service, or plugins whose
 * allocator belongs to someone else. Takes the same x, n, block, out and stream as
 * tgcb_sum_pairwise_f32 and gives the same result, but uses a scratch array built into the
 * library (TGCB_NOALLOC_SCRATCH_BYTES per device, held by every GPU that loads the library
 * until the process exits) instead of caller scratch, and calls no allocator.
 *   - Limit: n must need at most TGCB_NOALLOC_SCRATCH_BYTES of scratch, see
 *     tgcb_sum_pairwise_scratch_bytes(n, block); at block 8 that is up to 9 * 2^25 - 1
 *     (301,989,887) values.
 *     Larger n is refused with TGCB_E_INVALID before anything is launched.
 *   - The array's device address is looked up with the device current by tgcb_init(device),
 *     which allocates a status word of its own; after it, calls on that device do no look-up.
 *     A caller that never calls tgcb_init gets the look-up in its first call on each device
 *     (which may load the library's module there); make that first call before any stream
 *     capture. Devices 0 .. 15, as for tgcb_init.
 *   - Every call shares the one array, so calls whose kernels overlap on the GPU (different
 *     streams, or different host threads) race; serialise them. Nothing in the array has to
 *     start at zero: each level of the tree writes every partial it later reads. */
#define TGCB_NOALLOC_SCRATCH_BYTES (1u << 20)
int tgcb_sum_pairwise_f32_noalloc(const float* x, uint64_t n, int block, float* out, void* stream);

/* Per-row symmetric int8 quantisation, bit-exact to quantize.symmetric_scheme + quantise
 * applied per row (tgc/analysis/quantize.py:90-128, 229-240): m = max|row| in float32,
 * scale = float((double)m / 127) (1.0f for an all-zero row), q = rint(x / scale) clamped to
 * [-128, 127]. Writes q[rows*cols] (int8) and scale[rows] (float32). */
int tgcb_quantise_rows_i8(const float* x, int64_t rows, int64_t cols, int8_t* q, float* scale, void* stream);

/* ---- Peer memory and the gradient all-reduce over NVLink (one process per GPU) ----
 * Replaces what tgc only models: the all-reduce of data-parallel gradients priced by
 * tgc/parallel/collective.py:76-113 (ring_time, ring_volume) after shard.row_parallel
 * (tgc/parallel/shard.py:39-123). Buffers are shared between the processes of one box with
 * CUDA IPC (plain peer mappings over NVLink/NVSwitch; no multicast objects). */
#define TGCB_MAX_PEERS 8
#define TGCB_PEER_SLOTS 4
#define TGCB_PEER_MAX_SEGMENTS 8
#define TGCB_PEER_HANDLE_BYTES 64
/* Flag words a peer group needs per rank (ready and done words of every slot and rank, and a
 * finished count per slot). */
#define TGCB_PEER_FLAG_WORDS (2 * TGCB_PEER_SLOTS * TGCB_MAX_PEERS + TGCB_PEER_SLOTS)

/* cudaMalloc `bytes`, zero them and export them: *ptr is the local address, handle
 * (TGCB_PEER_HANDLE_BYTES) opens the same memory in another process of the box. */
int tgcb_peer_alloc(size_t bytes, void** ptr, void* handle);
/* cudaFree a buffer from tgcb_peer_alloc (NULL: nothing). Close it in every other process first. */
int tgcb_peer_free(void* ptr);
/* Map another process's buffer into this one (peer access enabled as needed). */
int tgcb_peer_open(const void* handle, void** ptr);
/* Unmap a buffer opened with tgcb_peer_open (NULL: nothing). */
int tgcb_peer_close(void* ptr);

/* One rank's view of a peer group: every rank's base address (this rank's own, the others'
 * from tgcb_peer_open) and every rank's flag words (TGCB_PEER_FLAG_WORDS zeroed words each). */
typedef struct tgcb_peer_group {
  int32_t rank;
  int32_t world;                   /* 1 .. TGCB_MAX_PEERS */
  void* bases[TGCB_MAX_PEERS];     /* 16-byte aligned */
  uint32_t* flags[TGCB_MAX_PEERS];
  uint64_t bytes;                  /* size of every rank's buffer at bases[r]: segments must lie inside */
} tgcb_peer_group;

/* float32 values at `offset` bytes (a multiple of 16) from every rank's base, `count` of them
 * (a positive multiple of 4). */
typedef struct tgcb_segment {
  uint64_t offset;
  uint64_t count;
} tgcb_segment;

/* Average the segments over the ranks, in place on every rank (what
 * dist.all_reduce(op=AVG) does, and what tgc's ring_time prices). Every rank calls it with
 * the same segments, slot, epoch and ctas; the epoch of a slot goes up by one per call,
 * starting at 1 (flags are never reset; 2^32 / ctas calls per slot). Rank r owns the r-th
 * share of the 16-byte vectors and, for each of them, adds the ranks' values in rank order
 * 0, 1, ..., divides by world and stores the result on every rank: the averages are
 * identical on all ranks and on every run. The kernel (ctas CTAs of 512 threads on `stream`)
 * ends when this rank's segments hold the averages. Calls in different slots may overlap.
 * Waits for other ranks are bounded (4 s): a rank that gives up records status 5 in the
 * device status word (tgcb_status) and returns. */
int tgcb_peer_allreduce_avg_f32(const tgcb_peer_group* g, const tgcb_segment* segs, int n_segs, int slot,
                                uint32_t epoch, int ctas, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TGCB_H_ */
