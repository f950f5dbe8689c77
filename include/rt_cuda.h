/*
 * rt_cuda.h -- C ABI of the B200 (sm_100a) Q4_K decode library, librtcuda.so.
 *
 * This is the drop-in boundary for rich-triplet's GPU decode path: every
 * entry point below replaces one function of the reference crate's Metal
 * surface (paths are relative to the reference crate root).  The reference's
 * own host language is Rust; its binding (an `extern "C"` block behind a
 * `cuda` cargo feature) needs only the plain pointers and sizes used here.
 *
 * Conventions
 *  - Every function returns RT_OK (0) or a negative RT_E_* status; nothing
 *    aborts the process.  rt_last_error() gives a one-line reason.
 *  - The caller owns host buffers; the library owns device buffers (rt_w,
 *    rt_dec).  A context owns one CUDA stream; every call on it is ordered on
 *    that stream.  A context is not thread-safe: use one per thread or GPU.
 *  - Weight matrices are [rows = out_features, cols = in_features], row-major,
 *    exactly as Q4KMat / MatBf16 hold them (src/autograd2.rs:1036-1042, 688-692).
 *  - flags: RT_HOST means x / y (or the source blob) are host pointers and the
 *    call returns when the result is in host memory; RT_DEVICE means they are
 *    device pointers and the call only enqueues work on rt_stream(ctx).
 */
#ifndef RT_CUDA_H
#define RT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------- */
#define RT_OK 0
#define RT_E_INVAL (-1)   /* bad argument (null pointer, unknown flag)      */
#define RT_E_CUDA (-2)    /* a CUDA runtime call failed                      */
#define RT_E_NOMEM (-3)   /* device or host allocation failed                */
#define RT_E_SHAPE (-4)   /* dimension mismatch or unsupported size          */
#define RT_E_FORMAT (-5)  /* weight format not accepted here                 */
#define RT_E_IO (-6)      /* file could not be read / is malformed           */
#define RT_E_STATE (-7)   /* call out of order (e.g. context full)           */
#define RT_E_TIMEOUT (-8) /* a bounded device-side wait gave up              */

/* ---- weight formats (values are GGUF tensor type ids, src/gguf_loader.rs:40-61;
 *      BF16 is GGUF type 30) ------------------------------------------- */
#define RT_FMT_F32 0
#define RT_FMT_Q4_0 2
#define RT_FMT_Q4K 12
#define RT_FMT_Q6K 14
#define RT_FMT_BF16 30

/* ---- pointer location flags ----------------------------------------- */
#define RT_HOST 0
#define RT_DEVICE 1

typedef struct rt_ctx rt_ctx; /* device + stream + last error          */
typedef struct rt_w rt_w;     /* a weight matrix resident in HBM        */
typedef struct rt_dec rt_dec; /* a Gemma 3 decode engine                */

/* ---- context ---------------------------------------------------------- */

/* Open `device` and create the context's stream.
 * Replaces the thread-local METAL_CTX set-up (src/metal_ops.rs:404-428). */
int rt_init(int device, rt_ctx** out);
void rt_destroy(rt_ctx* ctx);
/* Last error message of `ctx` ("" when none); never NULL. */
const char* rt_last_error(const rt_ctx* ctx);
const char* rt_version(void);
/* The cudaStream_t every call on ctx is ordered on (as void*). */
void* rt_stream(rt_ctx* ctx);
int rt_sync(rt_ctx* ctx);

/* ---- weights ---------------------------------------------------------- */

/* Copy a weight matrix to HBM in `fmt` (RT_FMT_Q4K: rows*cols/256*144 bytes;
 * RT_FMT_BF16: rows*cols*2; RT_FMT_F32: rows*cols*4).  Q4_K needs cols % 256 == 0,
 * BF16 needs cols % 8 == 0.
 * Replaces the weight upload + cache of metal_gemv_q4k_t / metal_gemv_bf16_t
 * (src/metal_ops.rs:811-815, 899-903) and MetalDecodeContext::new's uploads
 * (src/metal_decode.rs:1002-1121). */
int rt_weight_upload(rt_ctx* ctx, int fmt, const void* host, uint64_t bytes, int64_t rows, int64_t cols,
                     rt_w** out);
/* Copy a weight's device bytes back (for bit-exact checks of conversions). */
int rt_weight_download(rt_ctx* ctx, const rt_w* w, void* host, uint64_t bytes);
int rt_weight_info(const rt_w* w, int* fmt, int64_t* rows, int64_t* cols, uint64_t* bytes);
const void* rt_weight_device_ptr(const rt_w* w);
void rt_weight_free(rt_ctx* ctx, rt_w* w);

/* ---- GEMV ------------------------------------------------------------- */

/* y[rows] = dequant(W[rows, cols]) . x[cols], f32 accumulation.
 * Replaces metal_gemv_q4k_t (src/metal_ops.rs:799-860) and the CPU
 * Q4KMat::gemv_mt it mirrors (src/autograd2.rs:1953-2035). */
int rt_gemv_q4k(rt_ctx* ctx, const rt_w* w, const float* x, float* y, int flags);
/* y[rows] = bf16(W[rows, cols]) . x[cols], f32 accumulation.
 * Replaces metal_gemv_bf16_t (src/metal_ops.rs:887-960) / MatBf16::gemv_mt
 * (src/autograd2.rs:954-1000). */
int rt_gemv_bf16(rt_ctx* ctx, const rt_w* w, const float* x, float* y, int flags);

/* Greedy LM-head step that allocates nothing.  No counterpart in the
 * reference: its LM head and argmax run inside the decode context, whose
 * buffers are created up front (src/metal_decode.rs:1002-1121).  It is for
 * callers that cannot call cudaMalloc at that point: a serving process that
 * has handed nearly all HBM to its own KV-cache pool, or a token loop that
 * cannot take cudaMalloc's implicit device synchronisation.
 *
 * Enqueues, on `stream` (a cudaStream_t; NULL = the legacy default stream) of
 * the CURRENT device: y_dev[r] = bf16(W[r, :]) . x_dev for the [rows, cols]
 * row-major BF16 matrix at w_dev, then *token_dev = the greedy token of y_dev
 * by sample_token's rule at temperature 0 (src/transformer4.rs:3036-3091: the
 * LAST row of the largest softmax probability; see GreedySlot in the
 * sources).  All four pointers are device memory the caller owns; w_dev and
 * x_dev 16-byte aligned; cols a multiple of 8.  Returns once the work is
 * enqueued.
 *
 * Scratch: no context, no cudaMalloc, no allocating library call.  The only
 * scratch is a file-scope device array (~1.3 MiB per device): for up to
 * RT_ARGMAX_STATIC_SLOTS CTAs a greedy slot each and an arrival counter, 32
 * partial row sums per warp, and a unit counter per 16-row tile for up to
 * RT_ARGMAX_STATIC_MAX_ROWS rows.  The counters must be zero when a launch
 * starts: they are zero at module load and every launch sets them back to
 * zero, also a launch in which a bounded device-side wait gave up.  Such a
 * launch writes *token_dev = -1 (the caller reads the token anyway, so this
 * is how a failure is reported); the next call starts clean.  rows beyond
 * RT_ARGMAX_STATIC_MAX_ROWS, cols beyond 2^20 and launches needing more than
 * RT_ARGMAX_STATIC_SLOTS CTAs are rejected with RT_E_SHAPE.
 * Setup: the first call on each device (with that device current) looks up
 * the scratch address (cudaGetSymbolAddress) and sets the kernel's
 * shared-memory limit.  Under CUDA's lazy module loading that first call is
 * also when the module loads and the array's device memory is reserved: make
 * it before any stream capture, and while memory for the array is still free.
 * Overlapping calls on one device (two streams, or two threads) share the
 * scratch and race: serialize them.
 * errbuf (may be NULL) receives a one-line reason on failure. */
#define RT_ARGMAX_STATIC_SLOTS 512
#define RT_ARGMAX_STATIC_MAX_ROWS 1048576
int rt_gemv_bf16_argmax_static(const void* w_dev, int64_t rows, int cols, const float* x_dev, float* y_dev,
                               int32_t* token_dev, void* stream, char* errbuf, size_t errlen);

/* C[m, N] = A[m, K] . dequant(W)^T for a Q4_K weight W [N, K] (K a multiple
 * of 256): the prompt-length GEMM of prefill.  Replaces Q4KMat::matmul_q4k_t
 * (src/autograd2.rs:1437-1457) and matmul_q4k_t_exact (:1507-1625).  A is bf16
 * row-major [m, K] (uint16 bits), C is f32 row-major [m, N].  flags RT_HOST:
 * host A and C, the call copies and waits; RT_DEVICE: device pointers (16-byte
 * aligned), enqueued on the context stream.  For m > 16 the tensor cores take
 * fp16: each row of A is scaled by a power of two into fp16's range (exact for
 * bf16 input), each dequantised weight is rounded to fp16 (relative error <=
 * 2^-11), and the scale is undone on the f32 result.  For m <= 16 a multi-row
 * GEMV streams W once for all rows: the fp16 rows of A are split into two int8
 * planes per 256 columns (error <= 1.6e-5 of the segment's largest magnitude)
 * and multiplied by the exact Q4_K weights (relative L2 about 3e-5 against
 * the exact product of those fp16 rows). */
int rt_gemm_q4k(rt_ctx* ctx, const rt_w* w, const void* a, int64_t m, float* c, int flags);
/* The same product for a BF16 weight W [N, K] (K a multiple of 256), such as
 * the tied LM head over several sequences' final hidden states: replaces
 * MatBf16::matmul_by_t with M > 1 (src/autograd2.rs:757-776, 954-1000). */
int rt_gemm_bf16(rt_ctx* ctx, const rt_w* w, const void* a, int64_t m, float* c, int flags);
/* QLinear::forward (src/qlinear.rs:83-111) for a Q4_K or BF16 weight W
 * [out, in]: y[t, out] = x[t, in] . dequant(W)^T + bias (add_bias_rows,
 * src/qlinear.rs:49-61), x and y f32 row-major, bias f32 [out] or NULL.
 * t == 1 runs the GEMV (x split into three int8 planes: f32-level accuracy);
 * t > 1 the product of rt_gemm_q4k / rt_gemm_bf16 over fp16 rows of x (scaled
 * by powers of two into fp16's range; relative error about 1e-4), on the
 * multi-row GEMV for Q4_K weights and t <= 16, else on the tensor cores.  flags RT_HOST: host x, bias and y, the call copies and waits;
 * RT_DEVICE: device pointers (x and y 16-byte aligned), enqueued on the
 * context stream.  RT_E_FORMAT for other weight formats. */
int rt_qlinear_forward(rt_ctx* ctx, const rt_w* w, const float* x, int64_t t, const float* bias, float* y, int flags);
/* The launch plan rt_gemm_q4k / rt_gemm_bf16 (and the many-sequence engines)
 * choose for an [m, k] x [n, k]^T product on a GPU with num_sms SMs, without
 * a GPU (no counterpart in the reference): out[0] the CTA tile (16: the
 * multi-row GEMV, Q4_K weights at m <= 16; 128: weight rows as the 128-row
 * operand, activations as the narrow one when m <= 64; 256: 256 x 256),
 * out[1] the split-K count (the multi-row GEMV's K parts), out[2] the
 * activation rows per tile, out[3] the K columns per split.  RT_E_SHAPE when
 * no plan exists.  The RT_GEMM_TILE / RT_GEMM_SPLITS / RT_GEMM_ROWS tuning
 * overrides apply. */
int rt_gemm_plan(int64_t m, int64_t n, int32_t k, int32_t num_sms, int32_t bf16_weights, int32_t* out);

/* GEMV throughput measurement (no counterpart in the reference, whose GEMV
 * test times nothing).  Captures one CUDA graph of `launches` GEMVs of the
 * same shape, launch i reading ws[i % nw] (a rotation over several weight
 * copies keeps them out of L2), x_dev -> y_dev (device memory, 16-byte
 * aligned), each launch chained to the previous one by programmatic
 * dependent launch; replays it `reps` times and writes the mean device time
 * per GEMV in microseconds.  ctas_per_sm 1: one CTA per SM (the plan
 * rt_gemv_q4k uses); 2: half-size CTAs, so that the next GEMV of the chain
 * streams its weights beside the previous one.  Synchronises the context.
 * fmt: RT_FMT_Q4K or RT_FMT_BF16, matching every weight. */
int rt_gemv_bench(rt_ctx* ctx, int fmt, const rt_w* const* ws, int nw, const float* x_dev, float* y_dev, int launches,
                  int ctas_per_sm, int reps, float* us_per_gemv);

/* ---- load-time conversions (bit-exact with the reference CPU code) ---- */

/* GGUF Q4_0 bytes of a [rows, cols] tensor -> Q4_K weight in HBM, as
 * decode_q4_0_to_q4mat + Q4KMat::from_q4mat do on the CPU
 * (src/gguf_loader.rs:282-350, src/autograd2.rs:1291-1320, 1171-1246).
 * flags: RT_HOST or RT_DEVICE for `q4_0`. */
int rt_convert_q4_0_to_q4k(rt_ctx* ctx, const void* q4_0, int64_t rows, int64_t cols, int flags, rt_w** out);
/* GGUF Q6_K bytes -> BF16 weight in HBM, as decode_q6k_to_f32 +
 * f32s_to_bf16_and_drop do (src/gguf_loader.rs:482-533, src/transformer4.rs:1084-1097). */
int rt_convert_q6k_to_bf16(rt_ctx* ctx, const void* q6k, int64_t rows, int64_t cols, int flags, rt_w** out);

/* ---- Gemma 3 decode engine -------------------------------------------- */

/* Config4 (src/transformer4.rs:51-80).  Layer i is global iff i % 6 == 5
 * (Config4::is_global_layer, :141-143). */
typedef struct {
    int32_t vocab_size;          /* rows of the tied embedding / LM head */
    int32_t hidden_size;
    int32_t num_hidden_layers;
    int32_t num_attention_heads;
    int32_t num_key_value_heads;
    int32_t head_dim;
    int32_t intermediate_size;
    int32_t sliding_window;      /* 0 = no window on local layers */
    float rope_theta_local;
    float rope_theta_global;
    float rope_freq_scale_local;
    float rope_freq_scale_global;
    float rms_norm_eps;
    float query_pre_attn_scalar;
} rt_gemma3_cfg;

/* One Gemma3Block's weights (src/transformer4.rs:146-170, 290-300, 1936-1950).
 * Projections are rt_w handles already in HBM (Q4_K); the decoder copies them
 * into its own fused layout, so the handles may be freed afterwards.  Norm
 * weights are host f32 arrays holding gamma as the kernels apply it,
 * out = x_hat * (1 + gamma) (the value GGUF stores minus one, as the loader
 * keeps it: src/transformer4.rs:870-968). */
typedef struct {
    const rt_w *q, *k, *v, *o, *gate, *up, *down;
    const float *attn_norm, *post_attn_norm, *pre_ffn_norm, *post_ffn_norm; /* [hidden]   */
    const float *q_norm, *k_norm;                                            /* [head_dim] */
} rt_gemma3_layer;

/* Build the decode engine: upload norms, fuse QKV and gate/up, allocate an f32
 * KV cache of max_ctx positions and capture one decode step as a CUDA graph.
 * `embed` is the BF16 [vocab, hidden] embedding, tied with the LM head.
 * Replaces MetalDecodeContext::new (src/metal_decode.rs:971-1254). */
int rt_decoder_create(rt_ctx* ctx, const rt_gemma3_cfg* cfg, const rt_gemma3_layer* layers, const rt_w* embed,
                      const float* final_norm, int32_t max_ctx, rt_dec** out);
void rt_decoder_destroy(rt_dec* dec);

/* Load seq_len rows of one layer's K and V cache, host f32 in the CPU cache's
 * layout [seq_len, n_kv_heads * head_dim] (Gemma3LayerKvCache,
 * src/transformer4.rs:1794-1810).  Replaces sync_kv_from_cpu
 * (src/metal_decode.rs:1366-1396), without the f16 narrowing. */
int rt_decoder_load_kv(rt_dec* dec, int32_t layer, const float* k, const float* v, int32_t seq_len);
/* Read seq_len rows of one layer's K and V cache back, same layout. */
int rt_decoder_read_kv(rt_dec* dec, int32_t layer, float* k, float* v, int32_t seq_len);

/* One token: embed `token` at absolute `position`, run every layer, append its
 * K/V at `position`, and write vocab_size f32 logits to host `logits`.
 * Replaces MetalDecodeContext::decode_step (src/metal_decode.rs:2028-2074). */
int rt_decoder_step(rt_dec* dec, int32_t token, int32_t position, float* logits);

/* Run `n` prompt tokens through the engine one position at a time starting at
 * start_pos, filling the KV cache, and write the last token's logits (may be
 * NULL).  Replaces the CPU prefill + sync_kv_from_cpu hand-off
 * (src/transformer4.rs:2103-2164, 2190-2212). */
int rt_decoder_prefill(rt_dec* dec, const int32_t* tokens, int32_t n, int32_t start_pos, float* last_logits);

/* The same prefill with every position of a piece at once (up to 512 per
 * piece, longer prompts in order): each projection is one tensor-core GEMM
 * over the piece's tokens (fp16 operands, f32 accumulation), each token
 * attends causally to the cache and the piece's earlier tokens, and every
 * token's K/V lands in the cache as with rt_decoder_prefill.  Writes the last
 * token's logits (may be NULL).  The GPU counterpart of the reference's CPU
 * prefill (src/transformer4.rs:2103-2164). */
int rt_decoder_prefill_gemm(rt_dec* dec, const int32_t* tokens, int32_t n, int32_t start_pos, float* last_logits);

/* m (1..64) consecutive positions start_pos.. of this sequence in one pass,
 * their K/V appended, logits of all m rows to host `logits` ([m][vocab], may
 * be NULL): MetalDecodeContext::decode_step_batch (src/metal_decode.rs:
 * 2079-2579, M <= 8 there), the verify step of speculative decoding. */
int rt_decoder_step_batch(rt_dec* dec, const int32_t* tokens, int32_t m, int32_t start_pos, float* logits);

/* Greedy decode entirely on the device: step i feeds the argmax of step i-1
 * (largest logit, ties to the higher index) back as its token.  Starts from
 * `first_token` at `start_pos`.  tokens_out (host, may be NULL) receives the n
 * argmax tokens.  With flags == RT_DEVICE the n graph launches are only
 * enqueued on rt_stream() (tokens_out must be NULL); with RT_HOST the call
 * waits.  The decode loop of generate_cached_streaming
 * (src/transformer4.rs:2245-2439) with sample_token at temperature 0. */
int rt_decoder_generate(rt_dec* dec, int32_t first_token, int32_t start_pos, int32_t n, int32_t* tokens_out,
                        int flags);

/* Enqueue, on rt_stream(), only the Q4_K GEMV launches of one decode step with
 * the step's own shapes, layouts and inputs (one per projection group and
 * layer), for timing the dominant kernel alone.  *n_launches and *bytes
 * receive the launch count and the algorithmic bytes they move. */
int rt_decoder_enqueue_q4k_gemvs(rt_dec* dec, int32_t* n_launches, uint64_t* bytes);

/* Device bytes held by the engine (weights + KV cache + activations).
 * Replaces print_metal_memory (src/metal_decode.rs:1285-1354). */
int rt_decoder_memory(const rt_dec* dec, uint64_t* bytes);
/* The engine's kernel launches per decode step. */
int rt_decoder_launches_per_step(const rt_dec* dec, int32_t* n);
/* Copy an internal activation vector of the last step to host (debugging and
 * tests): which = 0 residual stream after the last layer, 1 logits, 2 the
 * phase timeline of the last persistent step kernel (1024 u64 globaltimer
 * stamps of CTA 0, read as 2048 f32 words; RT_E_INVAL when the engine runs
 * per-projection kernels), 3..7 the last layer's qkv, attention output, O
 * projection, gated FFN hidden and down projection.  `count` is the number of
 * f32 values to copy. */
int rt_decoder_read_activation(rt_dec* dec, int32_t which, float* host, int64_t count);

/* ---- many-sequence decode ----
 * The reference decodes one sequence per step; its decode_step_batch
 * (src/metal_decode.rs:2079-2579) batches positions of ONE sequence.  An
 * rt_batch advances `nseq` independent sequences per step on the weights of
 * an existing decoder (shared, not copied), each with its own f32 KV cache of
 * `cap` positions: every projection is one tensor-core GEMM over the
 * sequences (bf16 activations, f32 accumulation), attention runs per
 * sequence, and the greedy token of each sequence feeds its next step.
 * Tokens and positions stay on the device between steps. */
typedef struct rt_batch rt_batch;
int rt_batch_create(rt_dec* dec, int32_t nseq, int32_t cap, rt_batch** out);
void rt_batch_destroy(rt_batch* batch);
/* Host arrays [nseq]: each sequence's next input token and its position. */
int rt_batch_set(rt_batch* batch, const int32_t* tokens, const int32_t* positions);
/* One step; logits (host [nseq][vocab]) and next_tokens (host [nseq]) may be
 * NULL.  Afterwards each sequence's token is its greedy argmax and its
 * position has advanced by one.  Waits for the step. */
int rt_batch_step(rt_batch* batch, float* logits, int32_t* next_tokens);
/* `steps` greedy steps from the current tokens and positions.  RT_DEVICE:
 * enqueue only; RT_HOST: wait and report errors. */
int rt_batch_generate(rt_batch* batch, int32_t steps, int flags);
/* Tensor-parallel many-sequence decode (the reference has
 * no multi-GPU path).  `shard` is this rank's decoder: the model with its
 * 1/nranks of the query and KV heads and of the FFN columns (a multiple of
 * 256 each), the full embedding, norms replicated.  Per layer the o and down
 * outputs are summed over the ranks by an NCCL all-reduce; the LM head covers
 * this rank's vocab slice (rt_batch_vocab_slice) and the greedy token comes
 * from an all-gather of every rank's best logit.  Every rank calls this
 * together with the same nccl_id (rt_nccl_unique_id on one rank, 128 bytes,
 * shared by the caller; unused when nranks == 1) and then drives the returned
 * engine with rt_batch_set / rt_batch_step / rt_batch_generate in step. */
int rt_nccl_unique_id(void* id_out);
int rt_tp_create(rt_dec* shard, const void* nccl_id, int32_t nranks, int32_t rank, int32_t nseq, int32_t cap,
                 rt_batch** out);
/* The vocab rows [v0, v0 + vr) whose logits this engine's steps return (the
 * whole vocabulary without tensor parallelism). */
int rt_batch_vocab_slice(const rt_batch* b, int32_t* v0, int32_t* vr);
/* Peer all-reduce for a tensor-parallel engine (no reference counterpart):
 * the per-layer sums of the o and down outputs then cross NVLink as stores
 * into every rank's buffer, one kernel per sum, instead of NCCL all-reduces.
 * Every rank calls rt_tp_peer_handle (64 bytes: the CUDA IPC handle of this
 * rank's buffer), the caller gathers the handles in rank order, and every rank
 * calls rt_tp_peer_open with the nranks * 64 bytes; the step is then captured
 * again with the peer kernel.  Each wait on a peer is bounded (2 s), after
 * which the engine reports RT_E_TIMEOUT from the step and stops waiting.
 * Needs 2 to 8 ranks in one process each, on GPUs that reach each other. */
int rt_tp_peer_handle(rt_batch* b, void* handle_out);
int rt_tp_peer_open(rt_batch* b, const void* handles);

/* Test hook, no reference counterpart: the peer all-reduce kernel run by
 * this process as rank 0 of two, with the second rank's buffer a local zeroed
 * allocation whose flag never rises.  *err_word receives the error word after
 * two calls (3 = kErrGridTimeout when the first call's bounded flag wait gave
 * up), *first_ms / *second_ms their device times: the first call waits about
 * 2 s, the second, seeing the error word, does not wait at all. */
int rt_test_peer_allreduce_lonely(rt_ctx* ctx, int* err_word, float* first_ms, float* second_ms);

/* Fill every sequence's cache with synthetic values (a seeded hash, unit
 * variance) and set every position to seq_len: the state a benchmark decodes
 * from without prefilling. */
int rt_batch_synth_kv(rt_batch* batch, uint64_t seed, int32_t seq_len);
int rt_batch_info(const rt_batch* batch, uint64_t* bytes, int32_t* launches_per_step);

/* ---- Qwen 3.5 decode engine ------------------------------------------- */

typedef struct rt_qwen35 rt_qwen35; /* a Qwen 3.5 hybrid DeltaNet / attention decode engine */

/* ConfigQwen35 (src/transformer_qwen35.rs:32-151).  Layer i is full
 * attention iff (i + 1) % full_attention_interval == 0 (:133-135), else Gated
 * DeltaNet.  rope_dim = head_dim * partial_rotary_factor (:144-146). */
typedef struct {
    int32_t vocab_size;
    int32_t hidden_size;             /* multiple of 256 */
    int32_t num_hidden_layers;
    int32_t num_attention_heads;     /* full-attention query heads */
    int32_t num_key_value_heads;
    int32_t head_dim;                /* <= 512 */
    int32_t linear_num_key_heads;    /* DeltaNet */
    int32_t linear_num_value_heads;  /* a multiple of linear_num_key_heads */
    int32_t linear_key_head_dim;     /* <= 256 */
    int32_t linear_value_head_dim;   /* divides 256 */
    int32_t linear_conv_kernel_dim;
    int32_t intermediate_size;       /* multiple of 256 */
    int32_t full_attention_interval;
    int32_t rope_dim;
    float rms_norm_eps;
    float rope_theta;
} rt_qwen35_cfg;

/* One Qwen35Block's weights (src/transformer_qwen35.rs:262-284, 622-634,
 * 849-853, 881-886).  Projections are Q4_K rt_w handles [out, in] already in
 * HBM (the engine copies them into its fused layout, so they may be freed
 * afterwards); vectors are host f32.  input_norm / post_attn_norm / q_norm /
 * k_norm hold gamma as (1 + gamma) applies it; norm_weight is the DeltaNet
 * output norm's weight, applied as it is.  The DeltaNet fields are read on
 * DeltaNet layers, q/k/v/o/q_norm/k_norm on full-attention layers. */
typedef struct {
    const rt_w *gate, *up, *down;                                /* [F, H], [F, H], [H, F] */
    const float *input_norm, *post_attn_norm;                   /* [H] */
    const rt_w *in_qkv, *in_z, *in_a, *in_b, *out_proj;         /* [2 nk kd + nv vd, H], [nv vd, H], [nv, H] x 2, [H, nv vd] */
    const float *conv1d_weight;                                 /* [2 nk kd + nv vd][conv_kernel] */
    const float *a_log, *dt_bias;                               /* [nv] */
    const float *norm_weight;                                   /* [vd] */
    const rt_w *q, *k, *v, *o;  /* q: [nq * 2 head_dim, H] (each head's query then its gate), k/v: [nkv head_dim, H], o: [H, nq head_dim] */
    const float *q_norm, *k_norm;                               /* [head_dim] */
} rt_qwen35_layer;

/* Build the engine: fuse each layer's projections that share an input into
 * one Q4_K matrix, upload the vectors, allocate the DeltaNet states (zero),
 * the conv1d histories and an f32 K/V cache of max_tokens positions per
 * full-attention layer.  `embed` is the BF16 [vocab, hidden] embedding, tied
 * with the LM head; the caller keeps it alive while the engine exists.
 * Replaces MetalDecodeContextQwen35::new (src/metal_decode_qwen35.rs). */
int rt_qwen35_create(rt_ctx* ctx, const rt_qwen35_cfg* cfg, const rt_qwen35_layer* layers, const rt_w* embed,
                     const float* final_norm, int32_t max_tokens, rt_qwen35** out);
void rt_qwen35_destroy(rt_qwen35* eng);
/* Zero every DeltaNet state and conv1d history (a new sequence; the K/V
 * caches are overwritten position by position). */
int rt_qwen35_reset(rt_qwen35* eng);
/* One token at `position` (the cached sequence length): every layer's
 * forward_cached, the final norm and the LM head; vocab_size f32 logits to
 * host `logits` (may be NULL).  The Qwen35Model decode loop's CPU step
 * (src/transformer_qwen35.rs:1124-1133) and MetalDecodeContextQwen35::decode_step. */
int rt_qwen35_step(rt_qwen35* eng, int32_t token, int32_t position, float* logits);
/* The device address of the last step's logits ([vocab_size] f32). */
int rt_qwen35_logits_device(rt_qwen35* eng, const float** out);

/* ---- synthetic inputs ---------------------------------------------------
 * Deterministic, counter-based (SplitMix64) generators for benchmarks and
 * tests; the same (seed, stream) always gives the same bytes, independent of
 * thread count.  Host-side, no GPU needed. */

/* Q4_K blocks: per block d = f16(U[1e-3,1e-2]), dmin = f16(U[0,5e-3]) (f16 by
 * Q4KMat::f32_to_f16), 8 scales + 8 mins U{0..63} packed by pack_scales, 128
 * quant bytes U{0..255}.  out: rows*cols/256*144 bytes. */
void rt_synth_q4k(uint64_t seed, uint64_t stream, int64_t rows, int64_t cols, uint8_t* out);
/* Rows [row0, row0 + nrows) x columns [col0, col0 + ncols) (multiples of 256)
 * of rt_synth_q4k(seed, stream, rows, cols) as a Q4_K matrix of its own: the
 * bytes of slicing the whole matrix, made without it (tensor-parallel shards). */
void rt_synth_q4k_slice(uint64_t seed, uint64_t stream, int64_t rows, int64_t cols, int64_t row0, int64_t nrows,
                        int64_t col0, int64_t ncols, uint8_t* out);
void rt_synth_normal_f32(uint64_t seed, uint64_t stream, int64_t n, float mean, float stddev, float* out);
/* Normal values rounded to BF16 (round to nearest even). */
void rt_synth_normal_bf16(uint64_t seed, uint64_t stream, int64_t n, float mean, float stddev, uint16_t* out);
void rt_synth_tokens(uint64_t seed, uint64_t stream, int64_t n, int32_t vocab, int32_t* out);
void rt_synth_bytes(uint64_t seed, uint64_t stream, int64_t n, uint8_t* out);

#ifdef __cplusplus
}
#endif
#endif /* RT_CUDA_H */
