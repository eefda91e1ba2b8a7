// kernels.h -- launch interface between the host engine (engine.cpp) and the sm_100a kernels.
// Every matrix is row-major; activations are token-major [rows][features].
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

typedef __half f16;

namespace act {

// message returned by act_last_error(NULL) (defined with the C ABI in engine.cpp)
void set_last_error(const std::string& msg);
// inference lora_linear on host buffers (act_lora_linear); throws std::invalid_argument for bad
// arguments, std::runtime_error for CUDA failures
void lora_linear(int device, const float* x, int64_t rows, int in, int out, int w_type, const void* w,
                 size_t w_bytes, const float* A, const float* B, int rank, float alpha, const float* magnitude,
                 float strength, float* y);

// ---------------------------------------------------------------------------------------
// GEMM:  C[m][n] = epilogue( sum_k A(m,k) B(n,k) ),  K = K1 (+ K2 second segment).
//   A(m,k): a_kmajor ? A[m*lda + k] : A[k*lda + m]
//   B(n,k): b_kmajor ? B[n*ldb + k] : B[k*ldb + n]
// The second segment appends K2 reduction columns from (A2, B2) with the same majors; it
// carries the LoRA rank block so the adapter path rides in the same tile loop.
enum EpiMode : int {
    EPI_STORE_F32 = 0,   // out_f32 = alpha*acc
    EPI_ACCUM_F32 = 1,   // out_f32 += alpha*acc
    EPI_ATOMIC_F32 = 2,  // atomicAdd(out_f32, alpha*acc)        (split-K reductions)
    EPI_RESID_F32 = 3,   // out_f32 = resid + alpha*acc
    EPI_STORE_F16 = 4,  // out_bf16 = alpha*acc
    EPI_GELU = 5,        // aux_bf16 = acc ; out_bf16 = gelu(acc)
    EPI_GELU_BWD = 6,    // out_bf16 = acc * gelu'(auxin) * colscale2[n]
    EPI_BIAS_F16 = 7,   // out_bf16 = acc + bias[n]
    EPI_GELU_D = 8,      // z = f16(acc): aux_bf16 = gelu'(z) ; out_bf16 = gelu(z)   (z itself not kept)
    EPI_GELU_BWD_D = 9,  // out_bf16 = acc * auxin(= gelu') * colscale2[n]
};

struct GemmArgs {
    int M = 0, N = 0, K1 = 0, K2 = 0;
    const f16* A1 = nullptr;
    const f16* A2 = nullptr;
    long lda1 = 0, lda2 = 0;
    const f16* B1 = nullptr;
    const f16* B2 = nullptr;
    long ldb1 = 0, ldb2 = 0;
    bool a_kmajor = true, b_kmajor = true;
    int splitk = 1;
    // epilogue
    int mode = EPI_STORE_F32;
    float alpha = 1.0f;
    const float* colscale = nullptr;   // acc *= colscale[n] (DoRA row factor of the output)
    void* out = nullptr;
    long ldo = 0;
    const float* resid = nullptr;      // EPI_RESID_F32
    long ldr = 0;
    f16* aux = nullptr;               // additionally store acc (after colscale) as f16
    long ldaux = 0;
    const f16* auxin = nullptr;       // EPI_GELU_BWD: pre-activation; EPI_GELU_BWD_D: gelu' of it
    long ldauxin = 0;
    const float* colscale2 = nullptr;  // EPI_GELU_BWD: DoRA factor of the producing projection
    const float* bias = nullptr;       // EPI_BIAS_F16
    const float* rope = nullptr;       // rotate column pairs n < rope_cols by position m % rope_T
    int rope_T = 1, rope_cols = 0;     //   ([rope_T][32] (cos, sin) table, 64-column heads; after aux)
    int nvalid = 1 << 30;              // columns >= nvalid are not written
    int mvalid = 1 << 30;              // rows >= mvalid are not written
    // Stream-K workspace of the 2-CTA kernel (null: whole tiles only).  sk_part holds
    // gemm_sk_part_floats(), sk_flag gemm_sk_flag_count() zero-initialised ints that every
    // launch leaves at zero.  Launches sharing a workspace must not overlap on the device.
    float* sk_part = nullptr;
    int* sk_flag = nullptr;
    // fp32 output modes (STORE / ACCUM / RESID): also store f16(out), row stride ldo
    f16* out_h = nullptr;
    // Q8_0 weights in place of B1 / B2 (tcgen05 2-CTA path; the B pointer of that segment stays
    // null): Bq the quants biased to unsigned (q + 128), laid out exactly as B would be ([N][K]
    // K-major or [K][N] MN-major, row stride ldb), Bd the f16 block scales of those quants,
    // transposed: one row per 32 quant columns, [cols / 32][rows] with row stride ldd (a weight
    // [out][in] keeps its scales as [in / 32][out]).  Each quant is multiplied by its scale on
    // the way into the MMA.
    const uint8_t* B1q = nullptr;
    const f16* B1d = nullptr;
    long ldd1 = 0;
    const uint8_t* B2q = nullptr;
    const f16* B2d = nullptr;
    long ldd2 = 0;
    // tcgen05 paths: rows of A1 / A2 present in memory (0: M).  The tensor maps end there, so
    // rows arows .. M-1 read as zero; with mvalid <= arows nothing past them is written.  Lets
    // a product with a few rows (a rank block) run on a whole tile.
    int arows = 0;
    // 2-CTA kernel: A2 (the rank block) is written by the kernel launched immediately before
    // this one on the same stream, and A1, B1, B2 and every epilogue input by kernels before
    // that.  The GEMM then starts streaming its first K segment while its predecessor still
    // runs, and waits for the predecessor's completion only before its first A2 load (whole-
    // tile schedules; a stream-K launch waits at its start).
    bool a2_from_prev = false;
};
long gemm_sk_part_floats(int num_sms);
int gemm_sk_flag_count(int num_sms);

void gemm(const GemmArgs& a, cudaStream_t s);                 // mma.sync path, any layout
bool gemm_tc_supported(const GemmArgs& a);                     // shapes the tcgen05 path takes
void gemm_tc(const GemmArgs& a, int* err, cudaStream_t s);     // tcgen05 / TMEM / TMA path
bool gemm_tc2_supported(const GemmArgs& a);                    // 2-CTA (cta_group::2) 256-row pair tiles
void gemm_tc2(const GemmArgs& a, int* err, cudaStream_t s);     // 256 columns when N allows, else 128
void gemm_tc2_width(const GemmArgs& a, int* err, cudaStream_t s, int width);  // width 256 or 128
// Rank-block products on tcgen05 (gemm_skinny.cu): C = alpha * A(M x K) B(K x nb), nb <= 64,
// split over K across CTAs.  ACC / ACC_T add C (or C^T) into an fp32 gradient with atomics;
// STORE writes f16 C, reducing the split-K partials of a tile inside a thread-block cluster.
enum { SKINNY_ACC = 0, SKINNY_ACC_T = 1, SKINNY_STORE = 2 };
struct SkinnyArgs {
    int M = 0, K = 0, nb = 0;
    const f16* A = nullptr;  // A(m, k): a_mn ? A[k * lda + m] : A[m * lda + k]
    long lda = 0;
    bool a_mn = false;
    const f16* B = nullptr;  // B(k, n): b_mn ? B[k * ldb + n] : B[n * ldb + k]
    long ldb = 0;
    bool b_mn = false;
    int kind = SKINNY_ACC;
    float alpha = 1.0f;
    void* out = nullptr;      // ACC: out[m * ldo + n]; ACC_T: out[n * ldo + m]; STORE: f16 out[m * ldo + n]
    long ldo = 0;
    int splits = 0;           // 0: about two CTAs per SM (STORE: a power of two <= 8)
    // A as a Q8_0 weight in place of A (A stays null): Aq the quants biased to unsigned (q + 128),
    // laid out as A would be (row stride lda bytes), Ad their f16 block scales, one row per 32
    // quant columns ([cols / 32][rows], row stride ldad), dequantised on the way into the MMA
    const uint8_t* Aq = nullptr;
    const f16* Ad = nullptr;
    long ldad = 0;
};
bool skinny_supported(const SkinnyArgs& a);
void skinny_gemm(const SkinnyArgs& a, int* err, cudaStream_t s);

// tcgen05 path with the tile shape chosen per problem: 2-CTA 256 x 256 tiles unless they need
// more waves over the SMs than 1-CTA 128 x 256 tiles (Q8_0 segments: 2-CTA only)
void gemm_tc_auto(const GemmArgs& a, int* err, cudaStream_t s);
// Q8_0 blocks of a [rows][cols] weight (rows of cols / 32 blocks of 34 bytes: fp16 d, int8
// q[32]) -> quants biased to unsigned, q + 128, [rows][cols] and f16 scales [cols / 32][rows]
void q8_0_split(const uint8_t* blocks, int rows, int cols, uint8_t* q, f16* d, cudaStream_t s);
// Q8_0 weight view -> f16: out[r][c] = (q[r * ldq + c] - 128) * d[(c / 32) * ldd + r], rounded to
// f16 (the values the fused path feeds the MMA), for the paths that take f16 weights
void q8_view_to_f16(const uint8_t* q, long ldq, const f16* d, long ldd, int rows, int cols, f16* out, long ldo,
                    cudaStream_t s);

// ---------------------------------------------------------------------------------------
// attention over token-major q/k/v (head h at columns h*64 .. h*64+63), head_dim 64.
struct AttnArgs {
    const f16* q = nullptr;
    const f16* k = nullptr;
    const f16* v = nullptr;
    long ldq = 0, ldk = 0, ldv = 0;
    int T = 0;           // queries per clip
    int Tk = 0;          // stored keys per clip
    int H = 0;
    int clips = 0;
    const int* nvalid = nullptr;  // per clip: keys >= nvalid masked (nullptr: none)
    int causal = 0;
    int zero_key = 0;             // add_zero_attn: implicit key with score 0 and value 0
    const float* rope = nullptr;  // [T][32] (cos, sin) pairs of the self-attention RoPE
    int rope_load = 0;            // 1: q/k arrive unrotated (rotate while staging); 0: pre-rotated
                                  // (either way dq / dk come back unrotated)
    float scale = 0.125f;
    f16* o = nullptr;
    long ldo = 0;
    float* lse = nullptr;         // [clips][H][T], log2 units
    // backward
    const f16* dout = nullptr;
    long lddo = 0;
    float* dvec = nullptr;        // [clips][H][T]  rowsum(dO * O)
    float* dq_acc = nullptr;      // [clips*T][ldq_acc] fp32, rotated frame, zeroed by caller
    long ldq_acc = 0;
    // tcgen05 backward: per (clip, head, 128-query block) turn counters, zeroed by the caller
    // ([clips][H][ceil(T/128)]); when given, the key blocks add their dQ tiles into dq_acc in
    // key-block order (each waits for its predecessors' adds), so the sum is reproducible
    int* dq_turn = nullptr;
    // mma.sync backward with a single key block (Tk <= 64, no RoPE): dQ is final inside one CTA,
    // so it is written straight as f16 (times the optional column factor dq_scale) to dq_h;
    // dq_acc is then not used and needs no zeroing
    f16* dq_h = nullptr;
    long lddq_h = 0;
    const float* dq_scale = nullptr;
    f16* dk = nullptr;
    f16* dv = nullptr;
    long lddk = 0, lddv = 0;
    const float* kscale = nullptr;  // DoRA factor applied to dk columns (nullable)
    const float* vscale = nullptr;  // DoRA factor applied to dv columns (nullable)
    // mma.sync backward only: split each key block's query blocks over qsplit CTAs; each leaves
    // its partial dK / dV in its own slice of dk_acc / dv_acc ([qsplit][clips*Tk][H*64]) and
    // attn_dkv_finish adds the slices in order and writes dk / dv.  For few keys (cross-attention)
    // this spreads the query loop over the GPU instead of one CTA per (key block, head, clip).
    int qsplit = 1;
    float* dk_acc = nullptr;
    float* dv_acc = nullptr;
};

void attn_fwd(const AttnArgs& a, cudaStream_t s);
// the same forward on tcgen05 (attention_tc.cu): pre-rotated q/k (rope_load 0), Tk >= 64
bool attn_fwd_tc_supported(const AttnArgs& a);
void attn_fwd_tc(const AttnArgs& a, int* err, cudaStream_t s);
void attn_bwd(const AttnArgs& a, cudaStream_t s);  // computes dvec itself
void attn_dvec(const AttnArgs& a, cudaStream_t s);  // dvec = rowsum(dO * O)
void attn_dkv_finish(const AttnArgs& a, cudaStream_t s);  // dk / dv (f16) from dk_acc / dv_acc
// the same backward on tcgen05 (attention_tc.cu): pre-rotated q/k, Tk >= 128; computes dvec itself
// and adds into dq_acc (zeroed by the caller) like attn_bwd
bool attn_bwd_tc_supported(const AttnArgs& a);
void attn_bwd_tc(const AttnArgs& a, int* err, cudaStream_t s);
// cross-attention over at most 64 keys per clip on tcgen05 (xattn_tc.cu): no RoPE, not causal,
// query-major.  The forward writes o and lse; the backward recomputes the softmax (no lse / dvec),
// writes dq_h (f16, times dq_scale) and, with dk_acc / dv_acc given, one fp32 dK / dV slice per
// 128-query block (qsplit must equal ceil(T / 128)) added into dk / dv by attn_dkv_finish.
bool xattn_tc_supported(const AttnArgs& a);
bool xattn_bwd_tc_supported(const AttnArgs& a);
void xattn_fwd_tc(const AttnArgs& a, int* err, cudaStream_t s);
void xattn_bwd_tc(const AttnArgs& a, int* err, cudaStream_t s);
// dq (f16) = unrotate(dq_acc) * qscale[col]
void attn_dq_finish(const AttnArgs& a, f16* dq, long lddq, const float* qscale, cudaStream_t s);

// ---------------------------------------------------------------------------------------
// element-wise / row kernels
// LayerNorm over rows of D (fp32 in), y = xhat*w + b (+ add[row / rows_per_clip]) -> f16.
void layernorm_fwd(const float* x, const float* w, const float* b, const float* add, int rows_per_clip,
                   f16* y, float* mean, float* rstd, int rows, int D, float eps, cudaStream_t s);
// dx (=|+=) LN'(dy) (+ extra); also dx_h = f16(dx * colscale).  dy fp32.
void layernorm_bwd(const float* dy, const float* x, const float* w, const float* mean,
                   const float* rstd, float* dx, int accumulate, const float* extra, f16* dx_h,
                   const float* colscale, int rows, int D, cudaStream_t s);
// dst_h = f16((x (+ extra)) * colscale); x updated with extra when given.
void residual_to_f16(float* x, const float* extra, f16* dst, const float* colscale, int rows, int D,
                      cudaStream_t s);
void f32_to_f16(const float* x, f16* y, long n, cudaStream_t s);
// GELU of the f16 pre-activation (A&S 7.1.26, gelu_as_pair): gact = gelu(z) and, with
// store_grad, z <- gelu'(z) in place (n a multiple of 8)
void gelu_fwd(f16* z, f16* gact, long n, int store_grad, cudaStream_t s);
// the same evaluation on f16 bit patterns, element by element (stand-alone check)
void gelu_check(const uint16_t* z, uint16_t* g, uint16_t* dg, long n, cudaStream_t s);

// Gradient scale of the backward.  The seed gradient (the MSE's or the cross entropy's) is
// multiplied by a power of two gscale so that the f16 backward operands sit well inside the
// f16 range (d loss / d out is O(1 / (T * latent)) before scaling); every product that writes an
// fp32 adapter gradient multiplies by 1 / gscale, which is exact.

// MelodyFlow inputs: x0[m][c] = ((1-t)noise + t clean) * rescale(t), vstar = clean - noise.
// On-device posterior draws: clean (holding the mean) += stddev (held in noise) * N(0,1), noise =
// N(0,1), from Philox4x32-10 keyed by seed, counted by (element pair, window0 + clip)
void mf_sample(float* clean, float* noise, int clips, long per_clip, uint64_t seed, uint64_t window0, cudaStream_t s);
// start[b] >= 0: noise holds the edit-bridge pivot and becomes (pivot - start*clean) / (1 - start)
void mf_inputs(const float* clean, const float* noise, const float* t, const float* start, int clips, int T,
               int lat, f16* x0, float* vstar, cudaStream_t s);
// loss[b] = mean((sqrt2*out - vstar)^2) ; dout = gscale * d loss / d out (f16, token-major)
// part: clips * 32 floats of scratch (partial sums)
void mf_loss(const float* out, const float* vstar, int clips, int T, int lat, float* loss, f16* dout,
             float* part, float gscale, cudaStream_t s);
// small fp32 linear for the timestep MLP: y[b][n] = act(sum_k x[b][k] W[n][k]); act 1 = SiLU
void linear_f32(const float* x, const float* W, float* y, int rows, int N, int K, int act,
                cudaStream_t s);
// DoRA: dg[n] += inv_gscale * sum_m a[m][n] * b[m][n] / colscale[n]^2  (a already includes
// colscale and the gradient scale; dg is the unscaled gradient)
// dora_colsum splits the rows into at most DORA_COLSUM_PARTS blocks (enough to fill the GPU for
// the column count; fixed for a shape, so the ordered sum of the parts is reproducible); part
// holds DORA_COLSUM_PARTS * N floats; count holds ceil(N / 256) zero ints (left at zero)
constexpr int DORA_COLSUM_PARTS = 64;
void dora_colsum(const f16* a, long lda, const f16* b, long ldb, int rows, int N, const float* colscale,
                 float* dg, float* part, int* count, float inv_gscale, cudaStream_t s);
// DoRA-rows of one projection, for the batched kernels below (src/ac/lora.h:62-79 and the
// hand-derived backward of that factorisation)
struct DoraJob {
    const float *A, *B, *m;   // adapter values: lora_A [r][in], lora_B [out][r], magnitude [out]
    const float* P;           // W A^T [out][RP]
    const float* base;        // ||W_o||^2 + in * 1e-12
    float *G, *Q, *nsq, *g;   // per-step factors: A A^T [r][r], B G [out][r], row norms^2, m / row norm
    float* dg;                // d loss / d g [out], accumulated by dora_colsum
    float* scr;               // [out + r * r]: dt3, then dG
    float *gm, *gB, *gA;      // gradients of magnitude, lora_B, lora_A
    f16* BD;                  // [out][RP]: f16(bd_scale * dt2 * B), the rank block of gA += BD^T W
    int r, RP, in, out;
    float s;
};
// Per-step factors of n projections (jobs in device memory): G = A A^T, Q = B G,
// nsq = base + 2s<P,B> + s^2<B,Q>, g = m / sqrt(nsq); dg = 0.  P must be computed first.
void dora_factors(const DoraJob* jobs, int n, int r, int max_out, cudaStream_t st);
// Backward tail of n projections once their dg is complete: gm += dg/sqrt(nsq);
// dt2 = 2s dnsq, dt3 = s^2 dnsq; gB += dt2 P + 2 dt3 Q; BD = f16(bd_scale * dt2 * B) (the product
// gA += BD^T W that consumes it multiplies by 1 / bd_scale); dG = B^T diag(dt3) B; gA += 2 dG A
void dora_tail(const DoraJob* jobs, int n, int r, int max_out, int max_in, float bd_scale, cudaStream_t st);

// refresh f16 working copies: dst[row*ldd + col] = src[row*cols + col] for row<rows, col<cols
struct CopyJob {
    const float* src;
    f16* dst;
    int rows, cols, ldd;
};
void refresh_f16(const CopyJob* jobs_dev, int njobs, int max_elems, cudaStream_t s);

// AdamW over the flat parameter buffer (TrainAccumulation::update semantics).
// norm_partials: >= 1024 doubles of scratch.  nonfinite: int counter (accumulates).
void adamw(float* value, float* m, float* v, float* grad, const uint8_t* decay_mask, long n,
           float inv_count, float clip, float lr, float beta1, float beta2, float eps, float decay,
           float bc1, float bc2, double* norm_partials, int* nonfinite, cudaStream_t s);

// One bounded wait (the tcgen05 kernels' flag wait) on `flag` until it holds 1, giving up after
// limit_ns nanoseconds with WAIT_PROBE_CODE recorded in *err (wait_probe.cu).
constexpr int WAIT_PROBE_CODE = 99;
void wait_probe(const int* flag, long long limit_ns, int* err, cudaStream_t s);

// Q8_0 blocks -> f16 (one-time weight binding) and fp32 (parity checks).
void q8_0_to_f16(const uint8_t* blocks, long nblocks, f16* out, cudaStream_t s);
void q8_0_to_f32(const uint8_t* blocks, long nblocks, float* out, cudaStream_t s);

// MusicGen: x[s][:] = sum_q emb_q[ids[q][s]] + pos[s]   (fp32 out)
void mg_embed(const int32_t* ids, int steps, int nq, const float* const* emb_dev, const float* pos,
              float* x, int D, int seqs, cudaStream_t s);
// Cross entropy of one codebook over every sample's scored rows: row r of n * sel is sample
// b = r / sel, step s = r % sel, whose logits (fp32) / dlogits (f16) row is b * T + row0 + s of a
// [n * T][card] matrix and whose target is targets[b * tgt_stride + s] (-1: skip);
// loss_acc[b] += ce / nsel (row terms through rowloss [n * sel], added per sample in row order);
// dlogits = gscale * (softmax - onehot) / nsel.  Rows of dlogits outside the scored ones are not
// written.
void mg_cross_entropy(const float* logits, int n, int sel, int T, int row0, int card, const int32_t* targets,
                      long tgt_stride, float inv_nsel, float* loss_acc, float* rowloss, f16* dlogits, float gscale,
                      cudaStream_t s);

}  // namespace act
