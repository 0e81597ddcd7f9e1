/*
 * fgw_mha.h -- C ABI of the B200 (sm_100a) paged multi-head-attention forward.
 *
 * One shared library, libfgw_mha.so, exports these entry points. Arguments are plain device
 * pointers, sizes and a CUDA stream handle passed as void*; no framework types cross the
 * boundary. Every call is asynchronous on the given stream and returns an fgw_status for
 * argument and launch errors; device-side errors (a bounded wait that gave up) are recorded in
 * the workspace header and read back with fgw_mha_read_error.
 *
 * Reference interfaces replaced (paths inside zhangwenhao91/FGW):
 *   fgw_mha_paged_fwd       the launch callable returned by build_kernel and invoked by
 *                           mha_paged_decode: operators/mha/kernels/mha_paged_decode_ascend_v7.py:471-473
 *                           (direct, one split), :495-498 (partial then merge), :570 (call site);
 *                           general route: mha_paged_decode_ascend_cube_general.py:186-187, 284-288.
 *   fgw_mha_partial         the split-KV `partial` prim_func: v7.py:225-315 (compiled at :488-490),
 *                           cube_general.py:192-222.
 *   fgw_mha_merge           the LSE-weighted `merge` prim_func: v7.py:317-371, cube_general.py:224-279.
 *   fgw_mha_workspace_size  the per-call Parts/LSE buffers the reference allocates as kernel outputs
 *                           (v7.py:116, 232-233; out_idx=[5, 6] at :489).
 *   fgw_mha_plan / fgw_mha_attend  the two halves of fgw_mha_paged_fwd, exposed like the reference
 *                           exposes its compiled kernels on the launch callable for isolated profiling
 *                           (v7_experimental.py:842-855: direct_kernel / partial_kernel / merge_kernel).
 *   fgw_mha_device_sm_count the core count the reference reads from the device properties
 *                           (v7.py:65-68, 104-107 `cube_core_num`).
 *   fgw_mha_choose_splits   the host-side split choice from the cache lengths before each launch:
 *                           operators/mha/general_split_cost_model.py:70-91 (`predict_us`,
 *                           `select_model_splits`), with the B200 model's features and weights.
 *   fgw_paged_cache_gather  the paged-cache gather pre-pass FGW pins from TileOPs and runs before attention
 *                           in its gather experiment: third_party/tileops_yyttt6/paged_cache_gather.py:108-232
 *                           (`_compile`), :44-104 (`_compile_generic`), :264-296 (`forward`); call site
 *                           benchmarks/mha/external_cache_gather.py:38-58.
 */
#ifndef FGW_MHA_H_
#define FGW_MHA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FGW_MHA_ABI_VERSION 5

#if defined(__GNUC__)
#define FGW_API __attribute__((visibility("default")))
#else
#define FGW_API
#endif

typedef enum fgw_status {
  FGW_OK = 0,
  FGW_ERR_INVALID_ARGUMENT = 1,    /* shape, dtype, pointer or alignment precondition failed */
  FGW_ERR_UNSUPPORTED = 2,         /* valid request this build does not implement */
  FGW_ERR_WORKSPACE_TOO_SMALL = 3, /* workspace_bytes < fgw_mha_workspace_size(...) */
  FGW_ERR_CUDA = 4,                /* a CUDA runtime/driver call or a launch failed */
  FGW_ERR_DEVICE_TIMEOUT = 5,      /* a device-side bounded wait gave up (read via fgw_mha_read_error) */
  FGW_ERR_NO_DEVICE = 6            /* no sm_100 device is current */
} fgw_status;

/* Element types. The attention entry points take FLOAT16 / BFLOAT16; FLOAT8_E4M3 is a cache type of the
 * paged-cache gather only (fgw_paged_cache_gather). */
typedef enum fgw_dtype { FGW_DTYPE_FLOAT16 = 0, FGW_DTYPE_BFLOAT16 = 1, FGW_DTYPE_FLOAT8_E4M3 = 2 } fgw_dtype;

/* Which kernel family runs the QK^T -> softmax -> PV body. */
typedef enum fgw_path {
  FGW_PATH_AUTO = 0,   /* decode kernel for short query blocks, tensor-core kernel otherwise */
  FGW_PATH_DECODE = 1, /* warp-level HBM-streaming kernel (any q_len; intended for q_len <= 8) */
  FGW_PATH_TENSOR = 2  /* tcgen05/TMEM kernel, 128-row query tiles */
} fgw_path;

/*
 * How the main launch divides the work between its persistent CTAs (the reference's task_assignment,
 * v7.py:112-113, 260-270, and its static host stream plan, operators/mha/static_schedule.py:48-80, 195-247).
 *   STRIDED:    whole work items (request, head, split, query block) in longest-request-first order. The decode
 *               kernel deals them dynamically: a counter in the workspace hands the next item to whichever CTA
 *               asks, so CTAs finish within one item of each other. The tensor kernels deal them in snake
 *               order: round r gives CTA i item r * grid + i (r even) or r * grid + grid - 1 - i (r odd).
 *   CONTIGUOUS: the KV tiles of all work items, laid end to end, are cut into one contiguous range per CTA
 *               of equal length (loads differ by at most one tile); an item cut between CTAs is computed in
 *               pieces whose partial results the CTA finishing last merges in the same launch.
 *   TAIL:       STRIDED for the full waves (the first floor(items / G) * G items, G = the programs), then
 *               CONTIGUOUS over the items of the last, partial wave only (the reference's tail plan,
 *               static_schedule.py:83-116 `make_tail_plan`): only those items are cut into pieces.
 *   AUTO:       decode path: STRIDED (concurrent CTAs then read the heads of the same tokens together). Tensor
 *               path with one split, PAIRS and HALVES kernels: CONTIGUOUS only when there are fewer work items
 *               than 2/3 of 148 programs (whole items would leave SMs idle), STRIDED otherwise.
 * CONTIGUOUS and TAIL apply with num_splits == 1 to the decode kernel and to the PAIRS and HALVES tensor kernels;
 * elsewhere the launch runs STRIDED (fgw_mha_resolve_schedule reports which).
 */
typedef enum fgw_schedule {
  FGW_SCHEDULE_AUTO = 0,
  FGW_SCHEDULE_STRIDED = 1,
  FGW_SCHEDULE_CONTIGUOUS = 2,
  FGW_SCHEDULE_TAIL = 3
} fgw_schedule;

/* Which tcgen05 kernel runs the tensor path (no reference counterpart: FGW chooses its Cube kernel by route).
 *   AUTO:   PAIRS for head_dim <= 128, SINGLE above.
 *   PAIRS:  two 128-row query tiles per work item sharing every K/V tile (head_dim <= 128).
 *   SINGLE: one 128-row query tile per work item, P through shared memory (any head_dim).
 *   HALVES: one query tile per work item, S double-buffered in TMEM, the softmax split by key halves over two
 *           warpgroups (head_dim <= 128).
 * A kernel that cannot serve the head_dim returns FGW_ERR_UNSUPPORTED. */
typedef enum fgw_tensor_kernel {
  FGW_TENSOR_KERNEL_AUTO = 0,
  FGW_TENSOR_KERNEL_PAIRS = 1,
  FGW_TENSOR_KERNEL_SINGLE = 2,
  FGW_TENSOR_KERNEL_HALVES = 3
} fgw_tensor_kernel;

/*
 * Tensor contract (same as the reference, operators/mha/README.md:5):
 *   q        [batch, q_len, heads, head_dim]      fp16/bf16, contiguous
 *   k_cache  [pool_rows, heads, head_dim]         same dtype, contiguous, read-only
 *   v_cache  [pool_rows, heads, head_dim]         same dtype, contiguous, read-only
 *   block_table   [batch, table_width] int32      physical page ids (trusted, not range-checked)
 *   cache_seqlens [batch] int32                   0 <= len <= table_width * page_size
 *   out      [batch, q_len, heads, head_dim]      same dtype as q, written
 * Logical token t of request b lives at pool row block_table[b, t / page_size] * page_size
 * + t % page_size. Causal masking is right-aligned: query row i sees the first
 * max(len - q_len + i + 1, 0) tokens. Rows that see no token are written as exact zeros.
 */
typedef struct fgw_mha_params {
  const void* q;
  const void* k_cache;
  const void* v_cache;
  const int32_t* block_table;
  const int32_t* cache_seqlens;
  void* out;
  int64_t pool_rows;
  int32_t batch;
  int32_t q_len;
  int32_t heads;
  int32_t head_dim;    /* 16..256, multiple of 16 */
  int32_t table_width;
  int32_t page_size;   /* positive multiple of 16 dividing pool_rows */
  int32_t dtype;       /* fgw_dtype */
  int32_t causal;      /* 0 or 1 */
  int32_t num_splits;  /* split-KV partitions per query block, >= 1 (1 = direct output) */
  int32_t grid_cap;    /* persistent CTAs for the main kernel; 0 = one per work item */
  int32_t path;        /* fgw_path */
  int32_t wait_budget_ms; /* device-side wait limit; 0 = default (2000 ms) */
  int32_t schedule;       /* fgw_schedule */
  int32_t tensor_kernel;  /* fgw_tensor_kernel */
  int32_t reserved[2];    /* must be zero */
} fgw_mha_params;

/* The B200 split cost model (version 3): latency prediction = sum of weights[i] x feature i over the ten
 * features (constant, decode serial tiles, tensor serial tiles, decode waves, tensor waves, has merge, splits,
 * merge rows x splits, longest partition excess, contiguous pieces per item), floored at floor_single_us (one
 * split) or floor_multi_us; the choice is the smallest candidate (1, 2, ..., 128, at most the table's 128-token
 * tiles) whose prediction is within max(tolerance x best, absolute_margin_us) of the best. The values ship in
 * fgw_b200/operators/mha/models/b200_general_split_cost_model.json. */
#define FGW_SPLIT_MODEL_FEATURES 10
typedef struct fgw_split_model {
  double weights[FGW_SPLIT_MODEL_FEATURES];
  double floor_single_us;
  double floor_multi_us;
  double tolerance;
  double absolute_margin_us;
} fgw_split_model;

typedef struct fgw_split_choice {
  int32_t splits;         /* the model's split count (0 when the lengths are out of range) */
  int32_t full_kv_cache;  /* 1 when every cache length equals the table capacity */
  int32_t min_length;
  int32_t max_length;
} fgw_split_choice;

/* ABI version of the loaded library (FGW_MHA_ABI_VERSION it was built with). */
FGW_API int fgw_mha_abi_version(void);

/* Human-readable name of a status code (static storage). */
FGW_API const char* fgw_mha_status_string(int status);

/* Streaming multiprocessors of a CUDA device (148 on B200). */
FGW_API int fgw_mha_device_sm_count(int device, int* sm_count);

/* Host-only (no device work, no CUDA call): checks the host copy of the cache lengths against the table capacity
 * (page_size x table_width) and chooses the split count with the B200 model, in one pass over the lengths.
 * Returns FGW_ERR_INVALID_ARGUMENT for lengths outside [0, capacity] (choice->min_length / max_length still
 * report them) or non-positive extents. */
FGW_API int fgw_mha_choose_splits(const fgw_split_model* model, const int32_t* host_lengths, int batch, int q_len,
                                  int heads, int head_dim, int page_size, int table_width, int sm_count,
                                  fgw_split_choice* choice);

/* Kernel path AUTO resolves to for these parameters (FGW_PATH_DECODE or FGW_PATH_TENSOR). */
FGW_API int fgw_mha_resolve_path(const fgw_mha_params* params, int* path);

/* Schedule the main launch takes for these parameters (FGW_SCHEDULE_STRIDED, _CONTIGUOUS or _TAIL): AUTO and
 * requests a kernel cannot serve resolved as fgw_mha_paged_fwd resolves them. */
FGW_API int fgw_mha_resolve_schedule(const fgw_mha_params* params, int* schedule);

/* Bytes of device workspace fgw_mha_paged_fwd / fgw_mha_partial need for these parameters. */
FGW_API int fgw_mha_workspace_size(const fgw_mha_params* params, size_t* bytes);

/* Full forward: direct output when num_splits == 1, otherwise split partials merged into the output (on
 * the decode path by the kernel itself, the CTA completing a row group's splits merging them; on the
 * tensor path by a merge launch), on `stream`.
 * `workspace` must be 256-byte aligned device memory of at least fgw_mha_workspace_size bytes.
 * The workspace header's error word is cleared at the start of every call. */
FGW_API int fgw_mha_paged_fwd(const fgw_mha_params* params, void* workspace, size_t workspace_bytes, void* stream);

/* Planning pass alone: clears the workspace error word, clamps cache lengths into table capacity
 * and orders requests by descending length for the persistent schedule. fgw_mha_paged_fwd runs it
 * first; callers timing the attention kernel by itself run it once, then fgw_mha_attend. */
FGW_API int fgw_mha_plan(const fgw_mha_params* params, void* workspace, size_t workspace_bytes, void* stream);

/* Attention kernel alone, over a workspace fgw_mha_plan has prepared: writes the output directly
 * when num_splits == 1, else the split partials (follow with fgw_mha_merge). */
FGW_API int fgw_mha_attend(const fgw_mha_params* params, void* workspace, size_t workspace_bytes, void* stream);

/* Split-KV partial only: writes FP32 per-split normalised outputs and base-2 LSEs into the
 * workspace, for fgw_mha_merge to combine. Requires num_splits >= 2. */
FGW_API int fgw_mha_partial(const fgw_mha_params* params, void* workspace, size_t workspace_bytes, void* stream);

/* LSE-weighted merge of the partials fgw_mha_partial left in `workspace` into params->out. */
FGW_API int fgw_mha_merge(const fgw_mha_params* params, void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of the library-owned scratch array fgw_mha_paged_fwd_static_ws uses (16 MiB per GPU). */
#define FGW_MHA_STATIC_WORKSPACE_BYTES (16u << 20)

/* Allocation-free forward, for callers that cannot allocate device memory where they run attention
 * (inside an allocator or memory-pool callback, in a serving loop that forbids allocator calls, or in a
 * plugin whose host owns all device memory). No counterpart in the reference, which allocates its
 * scratch per call. Same kernels as fgw_mha_paged_fwd, but the workspace is a file-scope device array
 * of FGW_MHA_STATIC_WORKSPACE_BYTES held by every GPU that loads the library until exit; nothing is
 * allocated or freed. When an FGW_SCHEDULE_AUTO request's contiguous-schedule partial slots would not
 * fit, it runs the strided schedule instead (results then agree with fgw_mha_paged_fwd within the
 * library's floating-point tolerance, not bit for bit). Returns FGW_ERR_WORKSPACE_TOO_SMALL when the
 * request still needs more than that size. Counters and the error word that must start at zero are
 * zeroed on the device by each call's first kernel. The first call on a device looks up the array's
 * device address on the current device and keeps it for the process (a cudaDeviceReset invalidates it: do
 * not call this entry point after one); make that first call before any stream capture. All calls
 * share the one array, so calls that overlap on the GPU (different streams, or threads) race:
 * serialise them. */
FGW_API int fgw_mha_paged_fwd_static_ws(const fgw_mha_params* params, void* stream);

/* Device-side status of fgw_mha_paged_fwd_static_ws calls on the current device, for callers that never see
 * the library array's address (no reference counterpart): synchronises `stream`, then reports the error word
 * and wait site of the array's workspace header like fgw_mha_read_error. Each static-workspace call clears
 * them first, so the status is that of the last call. Allocates nothing. */
FGW_API int fgw_mha_static_ws_read_error(void* stream, int* device_status, int* site);

/* Synchronises `stream`, then reports the device-side status recorded in the workspace header
 * (FGW_OK or FGW_ERR_DEVICE_TIMEOUT) and which wait site gave up (0 when clean). */
FGW_API int fgw_mha_read_error(const void* workspace, void* stream, int* device_status, int* site);

/* Self-test of the device-side failure detection (no reference counterpart). One thread clears the
 * workspace header, then waits, with the same bounded wait every kernel of this library uses, on an
 * mbarrier phase that nothing completes (complete == 0) or that it completed itself first (complete != 0).
 * When `budget_ms` runs out the wait records FGW_ERR_DEVICE_TIMEOUT at site 99 and the kernel returns:
 * no trap, no fault, the context stays usable. Read the outcome with fgw_mha_read_error.
 * `workspace` needs the 256-byte header only. */
FGW_API int fgw_mha_selftest_wait(void* workspace, size_t workspace_bytes, int budget_ms, int complete,
                                  void* stream);

/*
 * Paged-cache gather: packs the cache rows that requests reach, in request order, into a dense buffer.
 * Output row r of request i (cu_seq_lens[i] <= r < cu_seq_lens[i + 1]) is the cache row
 *   block_table[i, pos / page_size] * page_size + pos % page_size,   pos = r - cu_seq_lens[i] + seq_starts[i]
 * (seq_starts NULL: 0). FLOAT16/BFLOAT16 rows are copied bit for bit (out_dtype == dtype); FLOAT8_E4M3 rows
 * become round_to_nearest(float(code) * scale[0]) in out_dtype (FLOAT16 or BFLOAT16). Rows before
 * cu_seq_lens[0] or from cu_seq_lens[batch] on, positions below 0 or past the table, and page ids outside
 * [0, num_pages) are written as zeros (the reference leaves them undefined); nothing is read out of bounds.
 * Offsets, starts, page ids and the scale stay device data. Asynchronous on `stream`.
 */
typedef struct fgw_gather_params {
  void* dst;                   /* [total_rows, row_width] out_dtype, contiguous, written */
  const void* cache;           /* [num_pages * page_size, row_width] dtype, contiguous, read-only */
  const int32_t* block_table;  /* [batch, table_width] physical page ids */
  const int32_t* cu_seq_lens;  /* [batch + 1] first output row of every request (non-decreasing) */
  const int32_t* seq_starts;   /* [batch] first logical position of every request, or NULL */
  const float* scale;          /* [1] dequantisation scale, FLOAT8_E4M3 caches only (NULL otherwise) */
  int64_t total_rows;          /* output rows (normally cu_seq_lens[batch]) */
  int32_t batch;
  int32_t num_pages;
  int32_t page_size;
  int32_t table_width;
  int32_t row_width;           /* elements per cache row (e.g. heads * head_dim) */
  int32_t dtype;               /* fgw_dtype of the cache */
  int32_t out_dtype;           /* fgw_dtype of dst: dtype, or FLOAT16/BFLOAT16 for an FP8 cache */
  int32_t reserved[3];         /* must be zero */
} fgw_gather_params;

FGW_API int fgw_paged_cache_gather(const fgw_gather_params* params, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FGW_MHA_H_ */
