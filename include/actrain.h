/*
 * actrain.h -- C ABI of the B200 adapter-training step (libactrain.so).
 *
 * This is the seam between the unchanged trainer front ends (mf-train / mg-train argument
 * parsing, cache sampling, checkpoint files) and the device step.  In the reference the
 * same seam is the class API of MfTrainGraph / MgTrainGraph plus TrainAccumulation:
 *   src/mf/train.h:31-256      MfTrainGraph  (ctor, compute, compute_bridge, adam_step, save)
 *   src/mg/train.h:51-230      MgTrainGraph  (ctor, compute, adam_step, save)
 *   src/ac/train_controls.h:75-119  TrainAccumulation (add, update)
 *   src/gguf_model.h:363-436   load_gguf / graph_compute_checked (weights on the device)
 *
 * Conventions: every call returns ACT_OK (0) or a nonzero status and never throws; the
 * message of the last failure is available from act_last_error().  A context is bound to
 * one CUDA device and is not thread-safe: one host thread per rank.  All pointers in the
 * batch structs are HOST pointers unless a name says otherwise.
 */
#ifndef ACTRAIN_H
#define ACTRAIN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define ACT_OK 0
#define ACT_ERR_INVALID 1    /* bad argument, shape or configuration (reference: std::runtime_error) */
#define ACT_ERR_CUDA 2       /* CUDA runtime failure */
#define ACT_ERR_NCCL 3       /* NCCL failure */
#define ACT_ERR_STATE 4      /* call out of order (e.g. step before act_finalize) */
#define ACT_ERR_NONFINITE 5  /* nonfinite loss or optimizer update (src/mf/train.h:186, train_controls.h:113) */

#define ACT_FAMILY_MELODYFLOW 0
#define ACT_FAMILY_MUSICGEN 1

#define ACT_ADAPTER_LORA 0
#define ACT_ADAPTER_DORA_ROWS 1

/* ggml type ids of the base weights accepted by act_bind_weight */
#define ACT_TYPE_F32 0
#define ACT_TYPE_F16 1
#define ACT_TYPE_Q8_0 8

/* adapter target bits, in the reference's order (src/mf/train.h:69, src/mg/train.h:90) */
#define ACT_TARGET_SELF_QKV (1u << 0)
#define ACT_TARGET_SELF_OUT (1u << 1)
#define ACT_TARGET_CROSS_Q (1u << 2)
#define ACT_TARGET_CROSS_KV (1u << 3)
#define ACT_TARGET_CROSS_OUT (1u << 4)
#define ACT_TARGET_FF0 (1u << 5)
#define ACT_TARGET_FF2 (1u << 6)
#define ACT_TARGETS_REFERENCE 0x1Fu     /* attention projections (default mf-train / mg-train) */
#define ACT_TARGETS_REFERENCE_FFN 0x7Fu /* with --train-ffn */

typedef struct act_ctx act_ctx;

/* Model hyper-parameters, read by the caller from GGUF metadata exactly as
 * DitConfig::from (src/mf/dit.h:44-71) and LmConfig::from (src/mg/lm.h:60-90) do. */
typedef struct {
    int family;                                  /* ACT_FAMILY_* */
    int dim, layers, heads, head_dim, ff_dim;
    int latent_dim, cond_dim, time_dim, n_skip;  /* MelodyFlow */
    int add_zero_attn;                           /* MelodyFlow */
    int n_q, card, special_token_id, pos_denominator; /* MusicGen */
    float max_period;                            /* MusicGen sin positions */
    float norm_eps;
} act_model_desc;

/* Adapter and capacity: MfTrainGraph(W, c, frames, tokens, rank, alpha, first_layer, seed,
 * type, feedforward) (src/mf/train.h:47-48) / MgTrainGraph(..., prefix, ...) (src/mg/train.h:66-67).
 * `targets` generalises the reference's feedforward flag (0x1F / 0x7F reproduce it). */
typedef struct {
    int type;          /* ACT_ADAPTER_LORA | ACT_ADAPTER_DORA_ROWS */
    int rank;
    float alpha;       /* scale = alpha / rank */
    int first_layer;
    unsigned targets;  /* ACT_TARGET_* bits */
    uint32_t seed;     /* lora_A ~ N(0, 0.02) drawn from std::mt19937(seed) in parameter order */
    int max_batch;     /* clips (MelodyFlow) or sequences (MusicGen) per step on this device */
    int frames;        /* latent frames (MelodyFlow) / codec timesteps (MusicGen) */
    int tokens;        /* conditioning tokens */
    int prefix_frames; /* MusicGen: timesteps before this are not scored (src/mg/train.h:195-196) */
} act_adapter_desc;

/* One MelodyFlow microbatch (MfTrainGraph::compute, src/mf/train.h:148-188), n <= max_batch. */
typedef struct {
    int n;
    const float* clean;        /* [n][latent_dim][frames] */
    const float* noise;        /* [n][latent_dim][frames] */
    const float* hidden;       /* [n][tokens][cond_dim] T5 states (zero padded) */
    const float* t;            /* [n] flow time in [0, 1] */
    const int32_t* unconditional; /* [n] or NULL: 1 masks every text token */
    const int32_t* valid_tokens;  /* [n] or NULL: tokens >= valid are masked; -1 = all */
    /* Edit-bridge objective (MfTrainGraph::compute_bridge, src/mf/train.h:190-204), or NULL for
     * flow matching.  The straight bridge x_t = (1-u) pivot + u clean, u = (t-start)/(1-start),
     * is trained through its equivalent t = 0 endpoint (pivot - start*clean) / (1 - start), which
     * the device forms in place of noise (noise may then be NULL).  Needs 0 <= start < 1 and
     * start <= t <= 1 for every sample. */
    const float* pivot;           /* [n][latent_dim][frames] */
    const float* edit_start;      /* [n] */
    /* On-device sampling (the reference draws these on the host, tools/mf-train.cpp:250-262):
     * when stddev is given, `clean` holds the posterior mean and the device draws clean = mean +
     * stddev * z and noise = z' (z, z' ~ N(0,1), Box-Muller from Philox4x32-10 keyed by
     * sample_seed, counted by window number window0 + i and element), and `noise` is ignored.
     * Reproducible per (seed, window, element), not the reference's host random stream.  Not
     * with pivot. */
    const float* stddev;          /* [n][latent_dim][frames] or NULL */
    uint64_t sample_seed;
    uint64_t window0;
} act_mf_batch;

/* One MusicGen microbatch (MgTrainGraph::compute, src/mg/train.h:178-227). */
typedef struct {
    int n;
    const int32_t* codes;      /* [n][n_q][frames] codec tokens in [0, card) */
    const float* context;      /* [n][tokens][dim] projected conditioning */
} act_mg_batch;

/* TrainAccumulation::update (src/ac/train_controls.h:89-118). */
typedef struct {
    float lr;            /* already scheduled: TrainControls::rate (src/ac/train_controls.h:53-58) */
    float beta1, beta2, eps;
    float weight_decay;  /* decoupled; applied to lora_A / lora_B only */
    float clip;          /* global L2 clip */
    int step;            /* 1-based optimizer step for bias correction */
    int count;           /* samples the gradient sum averages over; 0 = accumulated count */
} act_opt;

/* replaces the MfTrainGraph / MgTrainGraph constructors (graph build + allocation) */
int act_create(act_ctx** out, int device, const act_model_desc* model, const act_adapter_desc* adapter);
/* replaces load_gguf's tensor upload (src/gguf_model.h:363-420); name = GGUF tensor name */
int act_bind_weight(act_ctx* ctx, const char* name, int ggml_type, const void* host, size_t bytes);
/* after every weight: checks completeness, DoRA row norms (src/ac/lora.h:11-32), parameter init */
int act_finalize(act_ctx* ctx);

/* parameter table in the reference order (src/mf/train.h:68-104): name, flat offset, shape */
int64_t act_param_count(act_ctx* ctx);
int act_param_tensor_count(act_ctx* ctx);
int act_param_tensor(act_ctx* ctx, int index, char* name, size_t name_cap, int64_t* offset,
                     int64_t* rows, int64_t* cols);
int act_set_params(act_ctx* ctx, const float* value, size_t n);
/* value, m, v (any may be NULL): what save() and the .state sidecar write */
int act_get_params(act_ctx* ctx, float* value, float* m, float* v, size_t n);
int act_set_moments(act_ctx* ctx, const float* m, const float* v, size_t n);
int act_get_grads(act_ctx* ctx, float* grad, size_t n);
int act_zero_grads(act_ctx* ctx);

/* forward + backward of one microbatch; gradients accumulate on the device (the reference's
 * compute() followed by TrainAccumulation::add).  loss_per_sample may be NULL. */
int act_mf_step(act_ctx* ctx, const act_mf_batch* batch, float* loss_per_sample);
int act_mg_step(act_ctx* ctx, const act_mg_batch* batch, float* loss_per_sample);

/* data parallelism (no counterpart in the reference, which trains on one device) */
int act_nccl_get_unique_id(void* id_128_bytes);
int act_nccl_init(act_ctx* ctx, const void* id_128_bytes, int nranks, int rank);
/* sum gradients over ranks; nccl_comm NULL uses the context's own communicator.
 * global_count becomes the averaging count of the next act_optimizer. */
int act_allreduce_grads(act_ctx* ctx, void* nccl_comm, int global_count);
/* The next step (act_mf_step / act_mg_step / act_run_staged) all-reduces the gradients inside
 * the step, over the context's communicator: each layer's gradients start their all-reduce as
 * soon as that layer's backward has been issued (DoRA: once, after the whole backward), on a
 * stream of their own that overlaps the remaining backward.  It takes the place of
 * act_allreduce_grads after the last microbatch of an accumulation; global_count becomes the
 * averaging count of the next act_optimizer.  0 cancels. */
int act_set_grad_sync(act_ctx* ctx, int global_count);
/* Bit-for-bit reproducible steps (1) or the default (0).  Every reduction of the step is
 * order-independent except the self-attention backward's dQ, whose key blocks add their tiles
 * into one fp32 accumulator as they finish; with 1 they add in key-block order (each waits for
 * its predecessors, bounded), which makes the whole step a pure function of its inputs at the
 * cost of about 1.5 ms per cfg-2 step (5%).  The trainer front ends turn it on: exact resume and
 * checkpoints that leave training unchanged depend on it. */
int act_set_deterministic(act_ctx* ctx, int enable);
/* Bound, in milliseconds, on NCCL initialisation and on every host wait for the device while
 * a communicator is live (0 = none, the default).  A rank that stalls or dies makes the others'
 * next wait expire: their communicator is aborted (ncclCommAbort) and the call returns
 * ACT_ERR_NCCL instead of blocking forever. */
int act_set_timeout(act_ctx* ctx, int64_t timeout_ms);

/* mean, clip, AdamW, zero gradients (TrainAccumulation::update).  *nonfinite receives the
 * number of nonfinite updated values; a nonzero count also returns ACT_ERR_NONFINITE. */
int act_optimizer(act_ctx* ctx, const act_opt* opt, int* nonfinite);

const char* act_last_error(act_ctx* ctx);
void act_destroy(act_ctx* ctx);

/* ---- measurement hooks (device-resident inputs, kernel timing) ---- */
void* act_stream(act_ctx* ctx);   /* the cudaStream_t every kernel of the context runs on */
/* copy a batch to the device (host->device), then run it from device memory */
int act_mf_stage(act_ctx* ctx, const act_mf_batch* batch);
int act_mg_stage(act_ctx* ctx, const act_mg_batch* batch);
int act_run_staged(act_ctx* ctx, float* loss_per_sample /* may be NULL: no device->host read */);
/* per-kernel-class timing of eagerly launched steps: 0 disables (steps use the CUDA graph) */
int act_set_profiling(act_ctx* ctx, int enable);
/* class 0 = dense projection GEMMs, 1 = attention fwd+bwd, 2 = everything else */
int act_kernel_stats(act_ctx* ctx, int cls, double* ms, double* flops, double* bytes, int64_t* launches);
int act_reset_kernel_stats(act_ctx* ctx);
/* algorithmic FLOPs of one step of n samples (2 per multiply-add) */
double act_step_flops(act_ctx* ctx, int n);
/* stand-alone projection GEMM on host buffers (tests and the kernel sweep): C[M][N] fp32 =
 * A[M][K] . B(n,k) with f16 A and B, B as [N][K] (b_mn_major 0) or [K][N] (1);
 * path 0 = automatic, 1 = mma.sync kernel, 2 = tcgen05 kernel, 3 = tcgen05 2-CTA (cta_group::2)
 * kernel (stream-K split of the tiles where whole tiles would leave the last round mostly
 * idle), 4 = the 2-CTA kernel with 128-column pair tiles, 5 = the 2-CTA kernel on whole
 * tiles only; when reps > 0 the GEMM is
 * re-run reps times back to back and *ms_per_call receives the mean device time */
int act_gemm_f16(int device, const void* A, const void* B, void* C, int M, int N, int K, int b_mn_major, int path,
                 int reps, float* ms_per_call);
/* The same with B given as the Q8_0 blocks (34 bytes each, tools/ac-quantize.cpp:161) of the
 * weight [N][K] (b_mn_major 0) or [K][N] (1), kept quantised on the device: the 2-CTA kernel's
 * converter warps dequantise each k-block in shared memory (paths 0, 3, 4, 5).  The MMA sees the
 * values act_q8_0_dequant gives, so C equals act_gemm_f16 on that dequantised B bit for bit when
 * both run the same tile schedule (paths 4 and 5). */
int act_gemm_q8_0(int device, const void* A, const void* Bq8, void* C, int M, int N, int K, int b_mn_major, int path,
                  int reps, float* ms_per_call);
/* stand-alone rank-block product (tests and the kernel sweep): C = alpha * A(M x K) B(K x nb),
 * nb <= 64, f16 A stored [M][K] (a_mn 0) or [K][M] (1), f16 B stored [nb][K] (b_mn 0) or
 * [K][nb] (1).  kind 0: C [M][nb] fp32 += result; kind 1: C [nb][M] fp32 += result transposed;
 * kind 2: C [M][nb] = the result rounded to f16 (returned as fp32).  splits 0 = automatic.
 * No reference counterpart: the reference evaluates these products as separate ggml mul_mat
 * nodes (src/ac/lora.h:34-95).  When reps > 0 the call is re-run reps times (kind 0/1 keep
 * accumulating) and *ms_per_call receives the mean device time. */
/* stand-alone check of the feed-forward activation: g = f16(gelu(z)), dg = f16(gelu'(z)) for
 * f16 z (A&S 7.1.26 GELU of src/ac/lora.h:97-110 and the derivative of that approximation),
 * evaluated element by element (direct = 1) or by the vectorised pass the training step runs,
 * which overwrites the pre-activation with gelu' (0); the two agree bit for bit. */
int act_gelu_f16(int device, const uint16_t* z, uint16_t* g, uint16_t* dg, int64_t n, int direct);
int act_rank_gemm_f16(int device, int kind, const void* A, const void* B, float* C, int M, int K, int nb, int a_mn,
                      int b_mn, float alpha, int splits, int reps, float* ms_per_call);
/* The same product with A read from a frozen weight given as its Q8_0 blocks (34 bytes each,
 * tools/ac-quantize.cpp:161): the weight is [M][K] (a_mn 0) or [K][M] (1) and stays quantised on
 * the device; the kernel's converter warps dequantise each k-block on its way into the MMA (the
 * DoRA products P = W A^T and BD^T W of the training step, src/ac/lora.h:62-79).  With the same
 * splits, C equals act_rank_gemm_f16 on the act_q8_0_dequant f16 values bit for bit. */
int act_rank_gemm_q8_0(int device, int kind, const void* Aq8, const void* B, float* C, int M, int K, int nb, int a_mn,
                       int b_mn, float alpha, int splits, int reps, float* ms_per_call);
/* stand-alone attention forward + backward on host buffers (tests and the kernel sweep):
 * token-major f16 q [clips*T][H*64], k/v [clips*Tk][H*64], dout like q; scale 1/8 (head_dim 64);
 * nvalid: per-clip valid key count or NULL; causal; zero_key = the prepended zero key of
 * src/ac/transformer.h:74-79; rope: [T][32] (cos, sin) pairs or NULL.  Outputs o (f16),
 * lse (fp32 [clips][H][T], base-2 log-sum-exp of the scaled scores), and, when dout is given,
 * dq (f16, like q), dk / dv (f16, like k).  ms_fwd / ms_bwd (nullable) receive device times. */
int act_attention(int device, const void* q, const void* k, const void* v, const void* dout, int clips, int T,
                  int Tk, int H, const int32_t* nvalid, int causal, int zero_key, const float* rope, void* o,
                  float* lse, void* dq, void* dk, void* dv, float* ms_fwd, float* ms_bwd);
/* ---- attention backward that allocates nothing (no counterpart in the reference) ----
 * For callers that must not call cudaMalloc / cudaFree: real-time hosts such as an audio
 * plug-in's processing thread (an allocation can block and synchronise the device), code
 * recording a CUDA graph under global stream capture (allocation is not permitted there), and
 * embedders that own all device memory through their own pool.  Same computation and layouts
 * as the backward half of act_attention, but every pointer is a DEVICE pointer on the calling
 * thread's current device (nvalid and rope too), o and lse come from a forward pass, and the
 * work is queued asynchronously on `stream` (NULL = the legacy default stream).
 * Scratch (the fp32 dQ accumulator and the per-row rowsum(dO*O)) lives in one fixed array of
 * ACT_NOALLOC_ATTN_SCRATCH_FLOATS floats (32 MiB) compiled into the library; every GPU that
 * loads the library holds it until the process exits.  A problem needing more than
 * clips*T*H*64 + clips*H*T <= ACT_NOALLOC_ATTN_SCRATCH_FLOATS floats is rejected with
 * ACT_ERR_INVALID.  The first call on each device looks up that device's copy of the array
 * (cudaGetSymbolAddress); make that first call before any stream capture, and do not reset the
 * device (cudaDeviceReset or a primary-context reset) afterwards: the looked-up address is kept
 * for the life of the process.  Every call uses the same array and zeroes the accumulator it
 * needs, so calls that overlap on the GPU (on different streams, or from different threads)
 * race: serialise them.  q, k, v, o, dout, dq, dk and dv must be 16-byte aligned, rope 8-byte,
 * lse and nvalid 4-byte; other pointers are rejected with ACT_ERR_INVALID before any work is
 * queued. */
#define ACT_NOALLOC_ATTN_SCRATCH_FLOATS (8L * 1024 * 1024)
int act_attention_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const float* lse,
                              const void* dout, void* dq, void* dk, void* dv, int clips, int T, int Tk, int H,
                              const int32_t* nvalid, int causal, int zero_key, const float* rope, void* stream);
/* Kernel family each launch of the steps issued so far went to, counted as the launches are
 * issued (a captured graph counts once, when it is captured).  counts[i] for i < n receives the
 * count of ACT_PATH_i. */
#define ACT_PATH_ATTN_FWD_TC 0   /* tcgen05 self-attention forward (attention_tc.cu) */
#define ACT_PATH_ATTN_FWD_MMA 1  /* mma.sync attention forward (attention.cu) */
#define ACT_PATH_ATTN_BWD_TC 2   /* tcgen05 self-attention backward */
#define ACT_PATH_ATTN_BWD_MMA 3  /* mma.sync attention backward */
#define ACT_PATH_GEMM_TC 4       /* tcgen05 projection GEMM (gemm_tc.cu) */
#define ACT_PATH_GEMM_MMA 5      /* mma.sync GEMM (gemm_mma.cu) */
#define ACT_PATH_RANK_TC 6       /* tcgen05 rank-block product (gemm_skinny.cu) */
#define ACT_PATH_RANK_MMA 7      /* rank-block product on the mma.sync GEMM */
#define ACT_PATH_XATTN_FWD_TC 8  /* tcgen05 cross-attention forward, <= 64 keys (xattn_tc.cu) */
#define ACT_PATH_XATTN_BWD_TC 9  /* tcgen05 cross-attention backward, <= 64 keys */
#define ACT_PATH_COUNT 10
int act_path_counts(act_ctx* ctx, int64_t* counts, int n);
/* Failure-path check of the device error word (no reference counterpart): one kernel runs the
 * tcgen05 kernels' bounded flag wait on a flag that nothing sets, gives up after limit_ns
 * (1 ns .. 10 s), records its code, and the call returns ACT_ERR_CUDA as a step would after a
 * timed-out wait.  The word is cleared when reported: the context stays usable. */
int act_wait_probe(act_ctx* ctx, int64_t limit_ns);
/* MusicGen: read back the staged delayed inputs ([n][n_q][frames + n_q - 1], build_pattern_sequence
 * of src/mg/pattern.h:64-76 without its last step) and the scored targets ([n][n_q][frames -
 * prefix_frames], src/mg/train.h:195-205) of the last act_mg_stage / act_mg_step. */
int act_mg_staged(act_ctx* ctx, int32_t* ids, size_t n_ids, int32_t* targets, size_t n_targets);
/* MelodyFlow: read back the clean / noise windows of the last act_mf_stage / act_mf_step as the
 * device holds them ([n][latent_dim][frames] each; after on-device sampling, the drawn values). */
int act_mf_staged(act_ctx* ctx, float* clean, float* noise, size_t n_values);
/* Q8_0 blocks (34 bytes: fp16 d, int8 q[32]; tools/ac-quantize.cpp:161) dequantised on the
 * device by the kernels act_bind_weight uses: out_f32 = d * q in fp32, out_f16 = that value
 * rounded to nearest-even f16 (the GEMM operand).  Either output may be NULL. */
int act_q8_0_dequant(int device, const void* blocks, int64_t nblocks, float* out_f32, uint16_t* out_f16);
/* kernels in the captured step graph for microbatch size n (-1 before the graph exists) */
int64_t act_graph_kernel_nodes(act_ctx* ctx, int n);

/* ---- adapter consumption (inference) ---- */
/* lora_linear (src/ac/lora.h:50-83) on host buffers: y [rows][out] (fp32) = W x with the adapter
 * applied as load_lora (src/ac/lora.h:113-170) configures it.  x [rows][in] fp32; W [out][in] of
 * ggml type ACT_TYPE_F32 / F16 / Q8_0 (w_bytes its size); A [rank][in], B [out][rank] fp32, or A
 * NULL for the bare projection; magnitude [out] (DoRA rows) or NULL (LoRA).
 *   LoRA: y = W x + (strength * alpha / rank) B A x
 *   DoRA: y' = (W x + s B A x) * m / sqrt(||W_o||^2 + in*1e-12 + 2s<W_o,(BA)_o> + s^2||(BA)_o||^2),
 *         s = alpha / rank; y = W x + strength (y' - W x)
 * W x runs on the tensor cores (f16 operands: x and F32 weights rounded to f16, Q8_0 dequantised
 * inside the GEMM for more than 128 rows), the rank-sized products in fp32.  in and out must be
 * multiples of 8 (32 for Q8_0), rank <= 64.  Failures: ACT_ERR_INVALID / ACT_ERR_CUDA, message
 * from act_last_error(NULL). */
int act_lora_linear(int device, const float* x, int64_t rows, int in, int out, int w_type, const void* w,
                    size_t w_bytes, const float* A, const float* B, int rank, float alpha, const float* magnitude,
                    float strength, float* y);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif /* ACTRAIN_H */
