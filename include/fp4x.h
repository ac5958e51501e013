/*
 * fp4x — C ABI of the B200 (sm_100a) decode-GEMV library behind the fp4x vLLM plugin.
 *
 * Every entry point takes device pointers, plain integer sizes/strides and a CUDA stream (as void*), launches
 * asynchronously on that stream and returns FP4X_OK or a negative status; on failure
 * fp4x_last_error_message() describes it.  Nothing here allocates device memory: calls that need scratch take
 * a workspace pointer and a counters pointer sized by fp4x_gemv_query().  Counter arrays must be zero before
 * their first use; the kernels leave them zero again, so one array can be reused by every stream-ordered call.
 * Calls that share a workspace or a counter array must not overlap on the GPU (use one per stream).
 *
 * Layouts are those of the reference kernel library `x/fp4x_kernels.py` (cited as K:<line>):
 *   activations  bf16 [M, K], row stride x_stride (elements), 16-byte aligned rows
 *   MXFP8        codes e4m3 [N, K] bytes, scales e8m0 [N, K/32] bytes               (K:9-29)
 *   W8 g64       codes int8 [N, K], scales fp32 [N, K/64]                           (K:116-144)
 *   W6 g32       low nibbles [N, K/2], high bit pairs [N, K/4], scales fp16 [N, K/32] (K:151-202)
 *   NVFP4        e2m1 pairs [N, K/2] (low nibble = even k), e4m3 scales [N, K/16], fp32 global scale (K:73-113)
 *   INT2         2-bit codes [N, K/4] (bit pairs ORDER), fp16 scales [N, K/group]   (K:304-364)
 *   BF16         bf16 [N, K]                                                        (K:32-47)
 * Outputs are [M, N] (row stride out_stride elements) in bf16, f16 or fp32 (out_dtype).
 * Decode shapes: 1 <= M <= 16.
 */
#ifndef FP4X_H_
#define FP4X_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define FP4X_OK 0
#define FP4X_ERR_INVALID_ARG (-1)  /* null pointer, bad dtype, M outside 1..16, ... */
#define FP4X_ERR_UNSUPPORTED (-2)  /* shape or alignment the kernels do not handle */
#define FP4X_ERR_WORKSPACE (-3)    /* workspace or counter array too small */
#define FP4X_ERR_CUDA (-4)         /* a CUDA runtime call failed */
#define FP4X_ERR_DEVICE (-5)       /* a kernel recorded a device-side error (bounded wait expired) */

/* output dtypes */
#define FP4X_BF16 0
#define FP4X_F16 1
#define FP4X_F32 2

/* weight formats (fp4x_gemv_query) */
#define FP4X_FMT_MX8 0
#define FP4X_FMT_W8 1
#define FP4X_FMT_W6 2
#define FP4X_FMT_NV4 3
#define FP4X_FMT_BF16 4
#define FP4X_FMT_INT2 5

/* library version (major*10000 + minor*100 + patch) */
int fp4x_version(void);

/* message describing the last failing call on this host thread ("" if none) */
const char* fp4x_last_error_message(void);

/* Diagnostic (no reference counterpart): number of kernels this library has launched, or recorded into a CUDA
 * graph under capture, since it was loaded (all devices and threads).  Read before and after capturing a step to
 * count the library's kernels per step. */
int64_t fp4x_launch_count(void);

/* Reads (and optionally clears) the device error word that bounded waits set when they give up.
 * Synchronizes `stream`.  Returns FP4X_OK when the word is zero, FP4X_ERR_DEVICE otherwise.
 * A kernel whose wait gave up may leave arrival counters mid-count.  Clearing a non-zero word therefore also zeroes
 * the library's static counters (those of fp4x_mx8_linear_noalloc); counter arrays the caller passed in must be
 * zeroed by the caller before they are used again. */
int fp4x_device_error(void* stream, int clear, int* code_out);

/* Test hook (no reference counterpart): launches one CTA that waits on an mbarrier no thread arrives on, through
 * the library's bounded wait with a limit of limit_ns (1e3..1e9); the wait gives up, records its code in the device
 * error word and the kernel returns, so the next fp4x_device_error reports FP4X_ERR_DEVICE.  Nothing faults. */
int fp4x_test_expire_wait(int64_t limit_ns, void* stream);

/* Test hook (no reference counterpart): writes `value` into static arrival counter `index` of the current device
 * (the scratch of fp4x_mx8_linear_noalloc), to reproduce what a wait that gave up leaves behind.  Synchronous. */
int fp4x_test_set_static_counter(int64_t index, int32_t value, void* stream);

/* Scratch needed by one GEMV-family call: workspace bytes and number of int32 counters.
 * fmt: FP4X_FMT_*; batch: number of matrices of a batched call (1 otherwise); group: INT2 scale group. */
int fp4x_gemv_query(int fmt, int64_t m, int64_t n, int64_t k, int64_t batch, int group, size_t* ws_bytes,
                    int64_t* n_counters);

/* Diagnostic (no reference counterpart): writes a one-line description of the launch plan the library would use for
 * a GEMV of this format and shape (panels, chunks, CTAs, stages, shared memory, scratch) into buf. */
int fp4x_plan_describe(int fmt, int64_t m, int64_t n, int64_t k, int64_t batch, int group, int whole, char* buf,
                       size_t len);

/* Replaces mx8_linear (K:65-66 -> _run K:50-62 -> _mx8 K:9-29). */
int fp4x_mx8_linear(const void* x, int64_t x_stride, const void* w, const void* s, void* out, int64_t out_stride,
                    int out_dtype, int64_t m, int64_t n, int64_t k, void* ws, size_t ws_bytes, int32_t* counters,
                    int64_t n_counters, void* stream);

/* MXFP8 GEMV that allocates nothing and takes no scratch (no counterpart in the reference).  It always runs the
 * register-decode split-K kernel; fp4x_mx8_linear sends M <= 16 at 8192 rows or more to the tensor-core kernel, so
 * the two agree to fp32 summation order.  For callers that cannot hand the library a workspace or allocate device
 * memory at call time, such as a host runtime without a caching allocator.  The split-K scratch is a static
 * device array of the library: 8 MiB of partial tiles and 32768 int32 arrival counters per device.  Shapes whose
 * plan needs more are rejected with FP4X_ERR_WORKSPACE.  The first call on each device resolves the scratch address
 * (cudaGetSymbolAddress), so make it before capturing any stream on that device.  The counters are zero when the
 * library loads and each completed call leaves them zero; after a call that reported FP4X_ERR_DEVICE (a bounded wait
 * gave up), fp4x_device_error(stream, 1, ...) zeroes them again.  All calls on one device share the scratch, so calls
 * that may run at the same time (other streams or threads, without ordering) race: order them on one stream. */
int fp4x_mx8_linear_noalloc(const void* x, int64_t x_stride, const void* w, const void* s, void* out,
                            int64_t out_stride, int out_dtype, int64_t m, int64_t n, int64_t k, void* stream);

/* Replaces bf16_linear (K:69-70 -> _bg K:32-47). */
int fp4x_bf16_linear(const void* x, int64_t x_stride, const void* w, void* out, int64_t out_stride, int out_dtype,
                     int64_t m, int64_t n, int64_t k, void* ws, size_t ws_bytes, int32_t* counters,
                     int64_t n_counters, void* stream);

/* Replaces nv4_linear (K:102-113 -> _nv4 K:73-99); gs is the fp32 global scale. */
int fp4x_nv4_linear(const void* x, int64_t x_stride, const void* wp, const void* s, float gs, void* out,
                    int64_t out_stride, int out_dtype, int64_t m, int64_t n, int64_t k, void* ws, size_t ws_bytes,
                    int32_t* counters, int64_t n_counters, void* stream);

/* Replaces w8_linear (K:147-148 -> _w8 K:116-135). */
int fp4x_w8_linear(const void* x, int64_t x_stride, const void* q, const void* s, void* out, int64_t out_stride,
                   int out_dtype, int64_t m, int64_t n, int64_t k, void* ws, size_t ws_bytes, int32_t* counters,
                   int64_t n_counters, void* stream);

/* Replaces w6_linear (K:270-271 -> _w6 K:151-176). */
int fp4x_w6_linear(const void* x, int64_t x_stride, const void* lo, const void* hi, const void* s, void* out,
                   int64_t out_stride, int out_dtype, int64_t m, int64_t n, int64_t k, void* ws, size_t ws_bytes,
                   int32_t* counters, int64_t n_counters, void* stream);

/* Replaces int2_logits (K:359-364 -> _int2_head K:304-325, ROW_SCALE off).  `out_bf16` (may be NULL) receives
 * a bf16 copy of the logits with the same strides. */
int fp4x_int2_logits(const void* x, int64_t x_stride, const void* p, const void* s, int group, void* out,
                     int64_t out_stride, int out_dtype, void* out_bf16, int64_t m, int64_t n, int64_t k, void* ws,
                     size_t ws_bytes, int32_t* counters, int64_t n_counters, void* stream);

/* One W8 matrix of a batched call (the 48 router gates of a decode step, P:258-272 with FP4X_GATE=w8). */
typedef struct fp4x_w8_item {
  const void* x;   /* bf16 [M, K], 16-byte aligned rows */
  const void* q;   /* int8 [N, K], 16-byte aligned */
  const void* s;   /* fp32 [N, K/64] */
  void* out;       /* [M, N] */
} fp4x_w8_item;

/* Bytes of the device table that describes `count` batched W8 matrices. */
size_t fp4x_w8_batch_table_bytes(int64_t count);

/* Builds the device table of a batched W8 call from a HOST array of `count` items (TMA descriptors of the codes
 * plus the pointers).  `table` is device memory of fp4x_w8_batch_table_bytes(count) bytes, 64-byte aligned.
 * Synchronous (one host-to-device copy); run it once, outside any stream capture. */
int fp4x_w8_batch_prepare(const fp4x_w8_item* items, int64_t count, int64_t n, int64_t k, void* table,
                          size_t table_bytes);

/* Runs the `count` independent W8 GEMVs of a prepared table in a single launch.
 * Scratch: fp4x_gemv_query(FP4X_FMT_W8, m, n, k, count). */
int fp4x_w8_linear_batched(const void* table, int64_t count, int64_t x_stride, int64_t out_stride, int out_dtype,
                           int64_t m, int64_t n, int64_t k, void* ws, size_t ws_bytes, int32_t* counters,
                           int64_t n_counters, void* stream);

/* Fused hyper-connection down projection (HCFused.down K:503-510 -> _hc_down K:438-467): W8 split-K GEMV of
 * x [M, K] by q [N, K]; di [M, N] = bf16(sum); bot [M, lr] = bf16(t * sigmoid(t)), t = bf16(di / hc).
 * Scratch: fp4x_gemv_query(FP4X_FMT_W8, m, n, k, 1). */
int fp4x_hc_down(const void* x, int64_t x_stride, const void* q, const void* s, void* di, void* bot, int64_t m,
                 int64_t n, int64_t k, int64_t lr, int64_t hc, void* ws, size_t ws_bytes, int32_t* counters,
                 int64_t n_counters, void* stream);

/* Fused hyper-connection up projection (HCFused.up K:519-526 -> _hc_up K:470-493): W8 GEMV of bot [M, K] by the
 * stream-interleaved rows qi [hc*H, K] (HCFused.interleave_up K:513-517); out [M, H] =
 * bf16(sum_s bf16(nrm[m, s*H + j] * bf16(sigmoid(bf16(g_s)))) / hc), streams summed pairwise.
 * Requires hc * bj == 16 or 32 and n a multiple of 64. */
int fp4x_hc_up(const void* bot, int64_t bot_stride, const void* qi, const void* si, const void* nrm,
               int64_t nrm_stride, void* out, int64_t m, int64_t n, int64_t k, int64_t hc, int64_t bj, void* stream);

/* The unfused W8 mixer route (P:231-247): down GEMV + cast, scaled SiLU, up GEMV on the original row order
 * (qu/su), gate-mean — four launches whose arithmetic equals fp4x_hc_down + fp4x_hc_up bit for bit.
 * g: bf16 scratch [M, n_up].  Scratch: fp4x_gemv_query(FP4X_FMT_W8, m, n_down, k, 1). */
int fp4x_hc_mixer_unfused(const void* x, int64_t x_stride, const void* qd, const void* sd, const void* qu,
                          const void* su, void* di, void* bot, void* g, void* out, int64_t m, int64_t n_down,
                          int64_t k, int64_t lr, int64_t hc, int64_t n_up, void* ws, size_t ws_bytes,
                          int32_t* counters, int64_t n_counters, void* stream);


/* ---------------------------------------------------------------------------------------------------------
 * LM heads
 * Top-C order is total: value descending, then index ascending.  Selected index lists are written in ascending
 * index order.  Rows are limited to V <= 262144 and C <= 4096.
 * --------------------------------------------------------------------------------------------------------- */

/* Scratch of fp4x_topk for m rows. */
int fp4x_topk_query(int64_t m, int64_t v, int64_t c, size_t* ws_bytes, int64_t* n_counters);

/* Exact top-c per row of fp32 values [m, v] (replaces torch.topk at P:318,377 on the coarse logits).
 * idx_out [m, c] int32; val_out [m, c] (may be NULL) receives the selected values. */
int fp4x_topk(const float* vals, int64_t ld, int64_t m, int64_t v, int64_t c, int32_t* idx_out, int64_t idx_ld,
              float* val_out, int64_t val_ld, void* ws, size_t ws_bytes, int32_t* counters, int64_t n_counters,
              void* stream);

/* Replaces refine_mx8_ (K:384-388 -> _refine_mx8 K:367-381): exact fp32 dots of the MXFP8 rows idx[m, c]
 * (int32, or int64 when idx64) with x[m]; out[m, idx[m, c]] = cast(value) when out != NULL (in place into the
 * coarse logits) and exact_out[m, c] = value when exact_out != NULL. */
int fp4x_refine_mx8(void* out, int64_t out_ld, int out_dtype, const void* x, int64_t x_ld, const void* idx, int idx64,
                    int64_t idx_ld, const void* w, const void* s, int64_t m, int64_t c, int64_t k, float* exact_out,
                    int64_t exact_ld, void* stream);

/* Replaces refine_nv4 (K:412-417 -> _refine_nv4 K:391-409): out[m, c] = gs * sum_k bf16(e2m1 * s) * x. */
int fp4x_refine_nv4(float* out, int64_t out_ld, const void* x, int64_t x_ld, const void* idx, int idx64, int64_t idx_ld,
                    const void* wp, const void* s, float gs, int64_t m, int64_t c, int64_t k, void* stream);

/* out[m] = the index (from idx) of the largest value in vals[m, 0:c]; equal values: the smaller index. */
int fp4x_argmax_candidates(const float* vals, int64_t ld, const int32_t* idx, int64_t idx_ld, int64_t m, int64_t c,
                           int32_t* out, void* stream);

/* Scratch of fp4x_fast_head / fp4x_draft_head. */
int fp4x_fast_head_query(int64_t m, int64_t v, int64_t k, int64_t c, int group, size_t* ws_bytes,
                         int64_t* n_counters);

/* The fast target head (P:370-378): INT2 coarse logits over v rows, exact top-c, exact MXFP8 rescore.
 * full_bf16 [m, v] (contiguous) receives coarse bf16 logits with the c exact values scattered in;
 * idx_out / exact_out / coarse_out [m, c] and argmax_out [m] are optional (NULL to skip). */
int fp4x_fast_head(const void* x, int64_t x_ld, const void* p, const void* s, int group, const void* w8,
                   const void* s8, int64_t m, int64_t v, int64_t k, int64_t c, void* full_bf16, int64_t full_ld,
                   int32_t* idx_out, float* exact_out, float* coarse_out, int32_t* argmax_out, void* ws,
                   size_t ws_bytes, int32_t* counters, int64_t n_counters, void* stream);

/* The draft head (P:315-327): INT2 coarse logits over the v draft rows, top-c, exact NVFP4 rescore
 * (idx_out [m, c] draft-row indices, vals_out [m, c] fp32).  When full_bf16 and ids (int64 [v], draft row ->
 * vocab id) are given, full_bf16 [m, full_ld] is filled with -inf and the c values are scattered at ids[idx]. */
int fp4x_draft_head(const void* x, int64_t x_ld, const void* p, const void* s, int group, const void* wp,
                    const void* sn, float gs, int64_t m, int64_t v, int64_t k, int64_t c, int32_t* idx_out,
                    float* vals_out, const int64_t* ids, void* full_bf16, int64_t full_ld, int64_t full_v, void* ws,
                    size_t ws_bytes, int32_t* counters, int64_t n_counters, void* stream);

/* Merge of a vocab-sharded head (no reference counterpart: the reference runs TP=1; this is the exchange step
 * after an all-gather of every shard's candidates).  coarse / exact / gidx are [parts][m][c] (gidx = global
 * vocab ids); writes the global top-c by coarse value (idx_out ascending, coarse_out optional, exact_out) and
 * argmax_out [m] = the exact argmax among them. */
int fp4x_head_merge(const float* coarse, const float* exact, const int32_t* gidx, int64_t parts, int64_t m, int64_t c,
                    int64_t v, int32_t* idx_out, float* coarse_out, float* exact_out, int32_t* argmax_out,
                    void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Decode step in one persistent launch (no reference counterpart: the reference launches one Triton kernel per
 * linear, and its decode step is a CUDA graph of those launches, x/fp4patch.py:158-272, README.md:77-79).
 * An ordered list of the GEMV-family ops of a step runs as one kernel with one CTA per SM: each op computes exactly
 * what its standalone entry point computes (same weights, rounding and fixed summation order), ops wait only for
 * the earlier ops whose buffers they read or overwrite, and the weight stream of later ops is loaded while earlier
 * ops finish.  M <= 8 tokens.
 * --------------------------------------------------------------------------------------------------------- */
#define FP4X_STEP_NV4 0      /* nv4_linear: x [M, k] -> out [M, n], gs global scale */
#define FP4X_STEP_W6 1       /* w6_linear: p0 = low nibbles, p1 = high bit pairs, s = fp16 scales */
#define FP4X_STEP_W8 2       /* w8_linear: p0 = int8 codes, s = fp32 scales */
#define FP4X_STEP_HC_DOWN 3  /* fp4x_hc_down: out = di [M, n], out2 = bot [M, lr] */
#define FP4X_STEP_HC_UP 4    /* fp4x_hc_up: x = bot, p0/s = interleaved up rows, nrm, out [M, n / hc] */
#define FP4X_STEP_MX8 5      /* mx8_linear: p0 = e4m3 codes, s = e8m0 scales */

typedef struct fp4x_step_op {
  int kind;                /* FP4X_STEP_* */
  const void* x;           /* bf16 [M, k] activations, row stride x_stride elements */
  int64_t x_stride;
  const void* p0;          /* weight plane 0 */
  const void* p1;          /* weight plane 1 (W6 high bit pairs), else NULL */
  const void* s;           /* scales */
  float gs;                /* NVFP4 global scale */
  void* out;               /* [M, n] (row stride out_stride elements, out_dtype) */
  void* out2;              /* HC down: bot */
  int64_t out_stride;
  int out_dtype;
  int64_t n, k;
  int64_t lr, hc, bj;      /* hyper-connection ops */
  const void* nrm;         /* HC up: normalized streams [M, n] */
  int64_t nrm_stride;
} fp4x_step_op;

/* Sizes for a step of `count` ops at m tokens: device op table (64-byte aligned), workspace, int32 counters.
 * serial != 0 makes every op also wait for the op before it (the order of a single stream); otherwise ops wait
 * only for the earlier ops whose buffers they read or overwrite. */
int fp4x_step_query(const fp4x_step_op* ops, int64_t count, int64_t m, int serial, size_t* table_bytes,
                    size_t* ws_bytes, int64_t* n_counters);

/* Plans the ops, orders them by their buffer hazards and writes the device op table (one synchronous copy; run it
 * outside stream capture).  The workspace and the zeroed counters belong to the step until fp4x_step_release; the
 * counters are left zero after every completed run.  Buffers named by the ops must stay allocated. */
int fp4x_step_prepare(const fp4x_step_op* ops, int64_t count, int64_t m, int serial, void* table, size_t table_bytes,
                      void* ws, size_t ws_bytes, int32_t* counters, int64_t n_counters);

/* Runs a prepared step on `stream` (one launch; capturable in a CUDA graph).  Runs of one step must not overlap. */
int fp4x_step_run(const void* table, void* stream);

/* Diagnostic (no reference counterpart): with trace non-NULL, later runs of the step write a timeline to it:
 * [CTAs][ops][8] globaltimer nanoseconds at which each CTA started the op, had its inputs, had staged them,
 * finished it, had its first weight stage, left its stage loop and finished its last split-K flush (0 where a CTA
 * has no work in the op; the last entry is unused).  trace = NULL turns it off. */
int fp4x_step_trace(const void* table, uint64_t* trace, int64_t entries);

/* Forgets a prepared step (host bookkeeping only). */
int fp4x_step_release(const void* table);

/* ---------------------------------------------------------------------------------------------------------
 * Weight preparation on the GPU (replaces the reference's torch quantizers and dequantizers, K:138-357, and the
 * lazy preparation of x/fp4patch.py:61-83, :206-214, :290-307).  Inputs are row-major [n, k] weights in fp32, bf16
 * or f16 (FP4X_IN_*); outputs are the packed layouts listed at the top of this file.
 * The reference evaluates `tensor / python_scalar` as an IEEE division on the CPU and as a multiplication by the
 * fp32 reciprocal on CUDA devices, which can move a group scale by one ulp: FP4X_DIV_IEEE reproduces the
 * reference run on the CPU, FP4X_DIV_RECIP the reference run on a CUDA device.
 * --------------------------------------------------------------------------------------------------------- */
#define FP4X_IN_F32 0
#define FP4X_IN_BF16 1
#define FP4X_IN_F16 2
#define FP4X_DIV_IEEE 0
#define FP4X_DIV_RECIP 1

/* Replaces quantize_w8 (K:138-144): q int8 [n, k], s fp32 [n, k/64]. */
int fp4x_quantize_w8(const void* w, int in_dtype, int64_t n, int64_t k, int8_t* q, float* s, int div_mode,
                     void* stream);

/* Replaces quantize_w6 with clip_search = 0 (K:179-202): lo [n, k/2], hi [n, k/4], s_f16 [n, k/32]. */
int fp4x_quantize_w6(const void* w, int in_dtype, int64_t n, int64_t k, int qmax, uint8_t* lo, uint8_t* hi,
                     void* s_f16, int div_mode, void* stream);

/* Largest |w| over `count` weights into *amax_out (device fp32): the first pass of quantize_nv4 (K:286-288), whose
 * global scale gs = max(amax / 6 / 448, 1e-30) is then formed on the host in double precision, as there. */
int fp4x_amax(const void* w, int in_dtype, int64_t count, float* amax_out, void* stream);

/* Replaces the packing pass of quantize_nv4 (K:289-300): p [n, k/2] (low nibble = even k), s e4m3 [n, k/16]. */
int fp4x_quantize_nv4(const void* w, int in_dtype, int64_t n, int64_t k, double gs, uint8_t* p, uint8_t* s,
                      int div_mode, void* stream);

/* Replaces quantize_int2 with fp16 scales (K:330-351): p [n, k/4], s_f16 [n, k/group], group 16 or 32. */
int fp4x_quantize_int2(const void* w, int in_dtype, int64_t n, int64_t k, int group, uint8_t* p, void* s_f16,
                       int div_mode, void* stream);

/* Replaces mx8_dequant (K:261-267): out fp32 [n, k] = e4m3 * 2^(s - 127). */
int fp4x_mx8_dequant(const uint8_t* w8, const uint8_t* s, int64_t n, int64_t k, float* out, void* stream);

/* Replaces dequant_nv4 (K:420-426): out fp32 [n, k] = e2m1 * e4m3 scale * gs. */
int fp4x_dequant_nv4(const uint8_t* p, const uint8_t* s, double gs, int64_t n, int64_t k, float* out, void* stream);

/* Replaces dequant_int2 (K:353-357): out fp32 [n, k] = (code - 1.5) * s. */
int fp4x_dequant_int2(const uint8_t* p, const void* s_f16, int group, int64_t n, int64_t k, float* out, void* stream);

/* Replaces the scale un-swizzle of the draft head's NVFP4 source (x/fp4patch.py:296): scales stored as 128-row x
 * 4-column tiles, [n/128][kb/4][32][4][4], to row-major [n][kb] (row 128a + 32d + c, column 4b + e). */
int fp4x_nv4_unswizzle_scales(const uint8_t* in, int64_t n, int64_t kb, uint8_t* out, void* stream);

/* Replaces HCFused.interleave_up's row gather (K:513-517) for one plane of row_bytes bytes per row:
 * out row (j * hc + s) * bj + t = in row s * (n / hc) + j * bj + t. */
int fp4x_interleave_rows(const void* in, int64_t row_bytes, int64_t n, int64_t hc, int64_t bj, void* out,
                         void* stream);

/* Diagnostic with no reference counterpart: a launch timeline.  While installed, every GEMV launch (register-decode
 * and tcgen05 kernels) takes the next record of `records` (device memory, `count` records of 16 uint64 words, in
 * launch order; under stream capture the record is fixed at capture time and rewritten by every replay).  Words
 * (globaltimer ns, latest over the launch's CTAs unless noted): 0 earliest CTA start, 1 latest CTA start, 2 return
 * from the wait for the previous launch, 3 activation rows landed in shared memory, 4 activations converted (NVFP4
 * tensor-core kernel: token maxima known), 5 first weight stage ready, 6 accumulation done, 7 the two k-groups'
 * sums combined, 8 cross-CTA partial sums combined, 9 outputs stored, 10 earliest return from the wait, 11-15
 * unused.  Words 7 and 8 stay 0 in the tensor-core kernels.  The caller sets words 0 and 10 to all ones and the
 * others to zero before the launches run.  fp4x_timeline_end uninstalls the buffer and returns the number of
 * records handed out. */
int fp4x_timeline_begin(void* records, int64_t count);
int64_t fp4x_timeline_end(void);

/* Addition with no reference counterpart: pull up to 16 byte ranges (a later op's packed weights) from HBM into L2
 * while the stream's current op computes.  Stream-ordered as a programmatic-dependent launch: it releases the next
 * launch at once and retires only after the stream's previous work, so it adds no wait to the chain.  n = 0 or
 * zero-sized ranges launch nothing. */
int fp4x_prefetch_l2(const void* const* ptrs, const int64_t* bytes, int n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FP4X_H_ */
