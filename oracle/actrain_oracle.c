/*
 * actrain_oracle.c -- CPU restatement of the audiocraft.cpp adapter training step.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product links, loads or calls this file; it
 * is the checker that the parity tests, the smoke check and bench.py's CPU-baseline leg
 * compare the CUDA path against.
 *
 * What it restates (paths relative to the audiocraft.cpp source tree):
 *   - MelodyFlow DiT training forward   src/mf/dit.h:105-212, src/mf/train.h:106-108,148-188
 *   - MusicGen LM training forward      src/mg/train.h:12-49,131,178-227
 *   - shared blocks                     src/ac/transformer.h:55-61,74-79,108-125,144-154
 *   - LoRA / DoRA-rows linear           src/ac/lora.h:11-32,50-83
 *   - training LayerNorm and GELU       src/ac/lora.h:86-110
 *   - optimizer                         src/ac/train_controls.h:53-58,89-118,
 *                                       src/mf/train.h:206-227
 *   - delay pattern, positions          src/mg/pattern.h:31-86, src/mg/lm.h:102-116
 *   - skip plan                         src/mf/dit.h:87-100
 *   - Q8_0 blocks                       ggml block_q8_0 as written by tools/ac-quantize.cpp:161
 * The reference differentiates its graph with ggml autodiff (src/mf/train.h:118); ggml is
 * not present, so every backward rule below is derived by hand from the forward it
 * mirrors.  Arithmetic is fp32 (double where the reference uses double).
 *
 * Layouts: every matrix is row-major; a weight ggml stores as ne=[in,out] is [out][in];
 * activations are token-major [tokens][features] (ggml [dim, seq]).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORA_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------------------ */
/* configuration structs shared with tests (ctypes mirrors them field for field)        */

typedef struct {
    int dim, layers, heads, head_dim, ff_dim, latent_dim, cond_dim, time_dim, n_skip;
    float norm_eps;
    int add_zero_attn;
} ora_dit_cfg;

typedef struct {
    int dim, layers, heads, head_dim, ff_dim, n_q, card, special_token_id, pos_denominator;
    float max_period, norm_eps;
} ora_lm_cfg;

typedef struct {
    int rank;
    float alpha;
    int dora;          /* 0 = lora, 1 = dora-rows */
    int first_layer;
    unsigned targets;  /* bit i: suffix i of {self.qkv,self.out,cross.q,cross.kv,cross.out,ff.0,ff.2} */
} ora_adapter;

/* ------------------------------------------------------------------------------------ */
/* dense helpers                                                                         */

/* Register-blocked fp32 matmul: a 4 x 24 micro-tile of C stays in 12 AVX2 registers across a
 * k-chunk of KB_ while B is streamed from a packed panel.  Every element of C is summed over k
 * in ascending order, chunk after chunk, whatever the thread count: results do not depend on
 * the OpenMP schedule.  (The arithmetic is what the reference's CPU backend does for a mul_mat
 * node; only the order of the additions is this file's own.) */
#define MR_ 4
#define NR_ 24
#define MB_ 64
#define NB_ 240
#define KB_ 256

static int imin(int a, int b) { return a < b ? a : b; }

#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
/* c[MR_][ldc] += a[MR_][lda] (k = 0..kc-1) . bp[kc][NR_] */
static void ukern(int kc, const float* a, int lda, const float* bp, float* c, int ldc) {
    __m256 c00 = _mm256_loadu_ps(c), c01 = _mm256_loadu_ps(c + 8), c02 = _mm256_loadu_ps(c + 16);
    __m256 c10 = _mm256_loadu_ps(c + ldc), c11 = _mm256_loadu_ps(c + ldc + 8), c12 = _mm256_loadu_ps(c + ldc + 16);
    __m256 c20 = _mm256_loadu_ps(c + 2 * ldc), c21 = _mm256_loadu_ps(c + 2 * ldc + 8),
           c22 = _mm256_loadu_ps(c + 2 * ldc + 16);
    __m256 c30 = _mm256_loadu_ps(c + 3 * ldc), c31 = _mm256_loadu_ps(c + 3 * ldc + 8),
           c32 = _mm256_loadu_ps(c + 3 * ldc + 16);
    for (int k = 0; k < kc; ++k) {
        const __m256 b0 = _mm256_loadu_ps(bp + k * NR_), b1 = _mm256_loadu_ps(bp + k * NR_ + 8),
                     b2 = _mm256_loadu_ps(bp + k * NR_ + 16);
        __m256 av = _mm256_broadcast_ss(a + k);
        c00 = _mm256_fmadd_ps(av, b0, c00); c01 = _mm256_fmadd_ps(av, b1, c01); c02 = _mm256_fmadd_ps(av, b2, c02);
        av = _mm256_broadcast_ss(a + lda + k);
        c10 = _mm256_fmadd_ps(av, b0, c10); c11 = _mm256_fmadd_ps(av, b1, c11); c12 = _mm256_fmadd_ps(av, b2, c12);
        av = _mm256_broadcast_ss(a + 2 * lda + k);
        c20 = _mm256_fmadd_ps(av, b0, c20); c21 = _mm256_fmadd_ps(av, b1, c21); c22 = _mm256_fmadd_ps(av, b2, c22);
        av = _mm256_broadcast_ss(a + 3 * lda + k);
        c30 = _mm256_fmadd_ps(av, b0, c30); c31 = _mm256_fmadd_ps(av, b1, c31); c32 = _mm256_fmadd_ps(av, b2, c32);
    }
    _mm256_storeu_ps(c, c00); _mm256_storeu_ps(c + 8, c01); _mm256_storeu_ps(c + 16, c02);
    _mm256_storeu_ps(c + ldc, c10); _mm256_storeu_ps(c + ldc + 8, c11); _mm256_storeu_ps(c + ldc + 16, c12);
    _mm256_storeu_ps(c + 2 * ldc, c20); _mm256_storeu_ps(c + 2 * ldc + 8, c21); _mm256_storeu_ps(c + 2 * ldc + 16, c22);
    _mm256_storeu_ps(c + 3 * ldc, c30); _mm256_storeu_ps(c + 3 * ldc + 8, c31); _mm256_storeu_ps(c + 3 * ldc + 16, c32);
}
#else
static void ukern(int kc, const float* a, int lda, const float* bp, float* c, int ldc) {
    for (int i = 0; i < MR_; ++i)
        for (int k = 0; k < kc; ++k) {
            const float av = a[(size_t)i * lda + k];
            for (int j = 0; j < NR_; ++j) c[(size_t)i * ldc + j] += av * bp[k * NR_ + j];
        }
}
#endif

/* C[M][N] (=|+=) alpha * A[M][K] . B[K][N]; k-ascending accumulation per element. */
static void mm_nn(int M, int N, int K, const float* A, int lda, const float* B, int ldb,
                  float* C, int ldc, float alpha, int accumulate) {
    const int nib = (M + MB_ - 1) / MB_, njb = (N + NB_ - 1) / NB_;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int ib = 0; ib < nib; ++ib)
        for (int jb = 0; jb < njb; ++jb) {
            const int i0 = ib * MB_, i1 = imin(M, i0 + MB_), j0 = jb * NB_, j1 = imin(N, j0 + NB_);
            const int nj = j1 - j0, npan = (nj + NR_ - 1) / NR_;
            static __thread float acc[MB_ + MR_][NB_];
            static __thread float bp[KB_ * NB_];
            static __thread float ap[MR_][KB_];
            for (int i = 0; i < i1 - i0; ++i) memset(acc[i], 0, sizeof(float) * NB_);
            for (int k0 = 0; k0 < K; k0 += KB_) {
                const int kc = imin(K, k0 + KB_) - k0;
                /* pack B[k0 .. k0+kc)[j0 .. j1) as npan panels of [kc][NR_], zero padded */
                for (int p = 0; p < npan; ++p) {
                    float* dst = bp + (size_t)p * kc * NR_;
                    const int jj = j0 + p * NR_, w = imin(NR_, j1 - jj);
                    for (int k = 0; k < kc; ++k) {
                        const float* src = B + (size_t)(k0 + k) * ldb + jj;
                        int j = 0;
                        for (; j < w; ++j) dst[k * NR_ + j] = src[j];
                        for (; j < NR_; ++j) dst[k * NR_ + j] = 0.0f;
                    }
                }
                for (int i = i0; i < i1; i += MR_) {
                    const int h = imin(MR_, i1 - i);
                    const float* a = A + (size_t)i * lda + k0;
                    int la = lda;
                    if (h < MR_) { /* ragged last rows: pad a copy with zero rows */
                        for (int r = 0; r < MR_; ++r)
                            for (int k = 0; k < kc; ++k) ap[r][k] = r < h ? A[(size_t)(i + r) * lda + k0 + k] : 0.0f;
                        a = &ap[0][0];
                        la = KB_;
                    }
                    for (int p = 0; p < npan; ++p)
                        ukern(kc, a, la, bp + (size_t)p * kc * NR_, &acc[i - i0][p * NR_], NB_);
                }
            }
            for (int i = i0; i < i1; ++i) {
                float* c = C + (size_t)i * ldc + j0;
                for (int j = 0; j < nj; ++j)
                    c[j] = (accumulate ? c[j] : 0.0f) + alpha * acc[i - i0][j];
            }
        }
}

static float* transpose(int R, int Cc, const float* X, int ldx) {
    float* T = (float*)malloc(sizeof(float) * (size_t)R * Cc);
    /* 32 x 32 blocks: both sides stay in cache lines */
#pragma omp parallel for collapse(2) schedule(static) if ((long)R * Cc > 65536)
    for (int r0 = 0; r0 < R; r0 += 32)
        for (int c0 = 0; c0 < Cc; c0 += 32)
            for (int r = r0; r < imin(R, r0 + 32); ++r)
                for (int c = c0; c < imin(Cc, c0 + 32); ++c) T[(size_t)c * R + r] = X[(size_t)r * ldx + c];
    return T;
}

/* C[M][N] = alpha * A[M][K] . B[N][K]^T  (Y = X W^T) */
static void mm_nt(int M, int N, int K, const float* A, int lda, const float* B, int ldb,
                  float* C, int ldc, float alpha, int accumulate) {
    float* Bt = transpose(N, K, B, ldb);
    mm_nn(M, N, K, A, lda, Bt, N, C, ldc, alpha, accumulate);
    free(Bt);
}

/* C[M][N] = alpha * A[K][M]^T . B[K][N]  (weight-gradient form) */
static void mm_tn(int M, int N, int K, const float* A, int lda, const float* B, int ldb,
                  float* C, int ldc, float alpha, int accumulate) {
    float* At = transpose(K, M, A, lda);
    mm_nn(M, N, K, At, K, B, ldb, C, ldc, alpha, accumulate);
    free(At);
}

static float* zalloc(size_t n) { return (float*)calloc(n ? n : 1, sizeof(float)); }

/* ------------------------------------------------------------------------------------ */
/* fp16 and Q8_0                                                                          */

static float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
    if (exp == 0) {
        if (man == 0) bits = sign;
        else { /* subnormal: renormalise */
            int e = -1;
            do { ++e; man <<= 1; } while (!(man & 0x400));
            man &= 0x3ff;
            bits = sign | (uint32_t)(127 - 15 - e) << 23 | man << 13;
        }
    } else if (exp == 31) bits = sign | 0x7f800000u | man << 13;
    else bits = sign | (exp + 112) << 23 | man << 13;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* float -> fp16, round to nearest even (IEEE conversion, as numpy astype(float16)). */
static uint16_t float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return sign | 0x7c00 | (ax > 0x7f800000u ? 0x200 : 0);
    if (ax >= 0x477ff000u) return sign | 0x7c00; /* rounds to >= 65520 -> inf */
    if (ax < 0x38800000u) {                      /* result subnormal or zero */
        if (ax < 0x33000000u) return sign;        /* < 2^-25 rounds to 0 */
        const uint32_t e = ax >> 23, m = (ax & 0x7fffff) | 0x800000;
        const int shift = 126 - (int)e;           /* 14 + (113 - e) */
        uint32_t r = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (r & 1))) ++r;
        return sign | (uint16_t)r;
    }
    uint32_t r = ((ax >> 13) - (112u << 10));
    const uint32_t rem = ax & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (r & 1))) ++r;
    return sign | (uint16_t)r;
}

ORA_API float ora_half_to_float(uint16_t h) { return half_to_float(h); }
ORA_API uint16_t ora_float_to_half(float f) { return float_to_half(f); }

/* Q8_0: 34-byte blocks {fp16 d; int8 q[32]}, value = d * q (ggml block_q8_0). */
ORA_API void ora_q8_0_dequant(const uint8_t* blocks, int64_t nblocks, float* out) {
#pragma omp parallel for schedule(static) if (nblocks > 4096)
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint8_t* blk = blocks + b * 34;
        const float d = half_to_float((uint16_t)(blk[0] | blk[1] << 8));
        for (int i = 0; i < 32; ++i) out[b * 32 + i] = d * (float)(int8_t)blk[2 + i];
    }
}

static float roundf_away(float v) { /* round half away from zero, as ggml's roundf */
    const float a = fabsf(v), fl = floorf(a);
    const float r = fl + floorf(2.0f * (a - fl));
    return v < 0 ? -r : r;
}

/* ggml quantize_row_q8_0_ref: d = amax/127, q = round(x / d) with the fp32 d. */
ORA_API void ora_q8_0_quant(const float* x, int64_t nblocks, uint8_t* out) {
    for (int64_t b = 0; b < nblocks; ++b) {
        const float* v = x + b * 32;
        float amax = 0;
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
        const float d = amax / 127.0f, id = d != 0 ? 1.0f / d : 0.0f;
        const uint16_t dh = float_to_half(d);
        uint8_t* blk = out + b * 34;
        blk[0] = (uint8_t)(dh & 0xff);
        blk[1] = (uint8_t)(dh >> 8);
        for (int i = 0; i < 32; ++i) blk[2 + i] = (uint8_t)(int8_t)roundf_away(v[i] * id);
    }
}

/* ------------------------------------------------------------------------------------ */
/* small host-side pieces of the step                                                     */

/* src/mf/dit.h:87-100: consume if idx > L/2, produce if idx < L/2 - 1, projection idx % n. */
ORA_API void ora_skip_plan(int idx, int layers, int n_skip, int* consumes, int* produces,
                           int* projection) {
    const double half = (double)layers / 2.0;
    *consumes = n_skip > 0 && (double)idx > half;
    *produces = n_skip > 0 && (double)idx < half - 1.0;
    *projection = *consumes ? idx % n_skip : 0;
}

/* src/ac/transformer.h:144-154 (float arithmetic, as the reference). */
ORA_API void ora_timestep_features(float t, int dim, float max_period, float* out) {
    const int half = dim / 2;
    for (int i = 0; i < dim; ++i) out[i] = 0.0f;
    for (int i = 0; i < half; ++i) {
        const float freq = expf(-logf(max_period) * (float)i / (float)half);
        const float arg = t * freq;
        out[i] = cosf(arg);
        out[half + i] = sinf(arg);
    }
}

/* src/mf/dit.h:216-218 */
ORA_API float ora_dit_input_rescale(float t) {
    return 1.0f / sqrtf(t * t + (1.0f - t) * (1.0f - t));
}

/* src/mg/lm.h:102-116: double phase, [cos | sin], [n][dim]. */
ORA_API void ora_sin_positions(int first, int n, int dim, int pos_denominator, float max_period,
                               float* out) {
    const int half = dim / 2;
    for (int t = 0; t < n; ++t) {
        const double pos = (double)(first + t);
        for (int i = 0; i < half; ++i) {
            const double phase = pos / pow((double)max_period, (double)i / (double)pos_denominator);
            out[(size_t)t * dim + i] = (float)cos(phase);
            out[(size_t)t * dim + half + i] = (float)sin(phase);
        }
    }
}

/* src/mg/pattern.h:45-50: timestep carried by codebook q at sequence step s, or -1. */
static int pattern_timestep(int q, int s, int timesteps) {
    if (s <= 0) return -1;
    const int t = s - 1 - q; /* delays[q] = q (src/mg/lm.h:85) */
    return (t >= 0 && t < timesteps) ? t : -1;
}

/* src/mg/pattern.h:64-86: [n_q][T] -> [n_q][S], S = 1 + T + max_delay. */
ORA_API void ora_pattern_build(int n_q, int timesteps, const int32_t* codes, int32_t special,
                               int32_t* seq) {
    const int S = 1 + timesteps + (n_q - 1);
    for (int q = 0; q < n_q; ++q)
        for (int s = 0; s < S; ++s) {
            const int t = pattern_timestep(q, s, timesteps);
            seq[(size_t)q * S + s] = t >= 0 ? codes[(size_t)q * timesteps + t] : special;
        }
}

ORA_API void ora_pattern_revert(int n_q, int timesteps, const int32_t* seq, int32_t special,
                                int32_t* codes) {
    const int S = 1 + timesteps + (n_q - 1);
    for (size_t i = 0; i < (size_t)n_q * timesteps; ++i) codes[i] = special;
    for (int q = 0; q < n_q; ++q)
        for (int s = 0; s < S; ++s) {
            const int t = pattern_timestep(q, s, timesteps);
            if (t >= 0) codes[(size_t)q * timesteps + t] = seq[(size_t)q * S + s];
        }
}

ORA_API void ora_pattern_mask(int n_q, int timesteps, uint8_t* mask) {
    const int S = 1 + timesteps + (n_q - 1);
    for (int q = 0; q < n_q; ++q)
        for (int s = 0; s < S; ++s)
            mask[(size_t)q * S + s] = pattern_timestep(q, s, timesteps) >= 0;
}

/* ------------------------------------------------------------------------------------ */
/* LayerNorm (src/ac/lora.h:86-93) and the A&S 7.1.26 GELU (src/ac/lora.h:97-110)        */

static void ln_fwd(int n, int D, const float* x, const float* w, const float* b, float eps,
                   const float* add, float* y, float* mu, float* rs) {
#pragma omp parallel for schedule(static) if (n > 64)
    for (int i = 0; i < n; ++i) {
        const float* xi = x + (size_t)i * D;
        float s = 0;
        for (int j = 0; j < D; ++j) s += xi[j];
        const float m = s * (1.0f / (float)D);
        float ss = 0;
        for (int j = 0; j < D; ++j) ss += (xi[j] - m) * (xi[j] - m);
        const float r = 1.0f / sqrtf(ss / (float)D + eps);
        mu[i] = m;
        rs[i] = r;
        for (int j = 0; j < D; ++j)
            y[(size_t)i * D + j] = (xi[j] - m) * r * w[j] + b[j] + (add ? add[j] : 0.0f);
    }
}

/* dx += d(LN)/dx . dy (weight and bias are frozen). */
static void ln_bwd(int n, int D, const float* x, const float* w, const float* mu, const float* rs,
                   const float* dy, float* dx) {
#pragma omp parallel for schedule(static) if (n > 64)
    for (int i = 0; i < n; ++i) {
        const float* xi = x + (size_t)i * D;
        const float* di = dy + (size_t)i * D;
        float s1 = 0, s2 = 0;
        for (int j = 0; j < D; ++j) {
            const float g = di[j] * w[j], xh = (xi[j] - mu[i]) * rs[i];
            s1 += g;
            s2 += g * xh;
        }
        s1 /= (float)D;
        s2 /= (float)D;
        for (int j = 0; j < D; ++j) {
            const float g = di[j] * w[j], xh = (xi[j] - mu[i]) * rs[i];
            dx[(size_t)i * D + j] += rs[i] * (g - s1 - xh * s2);
        }
    }
}

static const float AS_P = 0.3275911f, AS_A1 = 0.254829592f, AS_A2 = -0.284496736f,
                   AS_A3 = 1.421413741f, AS_A4 = -1.453152027f, AS_A5 = 1.061405429f;

static float sgnf(float v) { return v > 0 ? 1.0f : v < 0 ? -1.0f : 0.0f; }

ORA_API float ora_gelu(float x) {
    const float z = x * 0.7071067811865475f, a = fabsf(z);
    const float t = 1.0f / (AS_P * a + 1.0f);
    const float poly = ((((AS_A5 * t + AS_A4) * t + AS_A3) * t + AS_A2) * t + AS_A1) * t;
    const float e = expf(-(z * z));
    const float erf_ = sgnf(z) * (1.0f - poly * e);
    return x * (0.5f * erf_ + 0.5f);
}

/* Derivative of the approximation itself (what autodiff of the op chain yields). */
ORA_API float ora_gelu_grad(float x) {
    const float z = x * 0.7071067811865475f, a = fabsf(z), sg = sgnf(z);
    const float t = 1.0f / (AS_P * a + 1.0f);
    const float poly = ((((AS_A5 * t + AS_A4) * t + AS_A3) * t + AS_A2) * t + AS_A1) * t;
    const float dpoly = (((5.0f * AS_A5 * t + 4.0f * AS_A4) * t + 3.0f * AS_A3) * t + 2.0f * AS_A2) * t + AS_A1;
    const float e = expf(-(z * z));
    const float erf_ = sg * (1.0f - poly * e);
    /* d erf / dz = sg*sg * dpoly * p t^2 * e + 2 z sg * poly * e */
    const float derf = sg * sg * dpoly * AS_P * t * t * e + 2.0f * z * sg * poly * e;
    return (0.5f * erf_ + 0.5f) + x * 0.5f * derf * 0.7071067811865475f;
}

/* ------------------------------------------------------------------------------------ */
/* attention (src/ac/transformer.h:74-79,108-125) with RoPE (src/ac/transformer.h:55-61)  */

typedef struct {
    int T, Tk, H, hd;   /* queries, stored keys, heads, head dim */
    int zero_key;       /* add_zero_attn: implicit key 0 with score 0 and value 0 */
    int causal;         /* key j > query i masked */
    int nvalid;         /* keys >= nvalid masked (the reference's -inf mask columns) */
    float scale;
} attn_shape;

/* q [T][ldq], k/v [Tk][ldk] (head h at column h*hd); o [T][ldo]; lse [H][T]. */
static void attn_fwd(const attn_shape* a, const float* q, int ldq, const float* k, int ldk,
                     const float* v, int ldv, float* o, int ldo, float* lse) {
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int h = 0; h < a->H; ++h)
        for (int i = 0; i < a->T; ++i) {
            float* s = (float*)malloc(sizeof(float) * (a->Tk + 1));
            const float* qi = q + (size_t)i * ldq + h * a->hd;
            float m = a->zero_key ? 0.0f : -INFINITY;
            int kend = a->nvalid < a->Tk ? a->nvalid : a->Tk;
            if (a->causal && kend > i + 1) kend = i + 1;
            for (int j = 0; j < kend; ++j) {
                const float* kj = k + (size_t)j * ldk + h * a->hd;
                float d = 0;
                for (int c = 0; c < a->hd; ++c) d += qi[c] * kj[c];
                s[j] = d * a->scale;
                if (s[j] > m) m = s[j];
            }
            float sum = a->zero_key ? expf(0.0f - m) : 0.0f;
            for (int j = 0; j < kend; ++j) { s[j] = expf(s[j] - m); sum += s[j]; }
            float* oi = o + (size_t)i * ldo + h * a->hd;
            for (int c = 0; c < a->hd; ++c) oi[c] = 0;
            for (int j = 0; j < kend; ++j) {
                const float p = s[j] / sum;
                const float* vj = v + (size_t)j * ldv + h * a->hd;
                for (int c = 0; c < a->hd; ++c) oi[c] += p * vj[c];
            }
            lse[(size_t)h * a->T + i] = m + logf(sum);
            free(s);
        }
}

/* dq [T][lddq] (=), dk/dv [Tk][..] (+=). Recomputes P from q, k and lse. */
static void attn_bwd(const attn_shape* a, const float* q, int ldq, const float* k, int ldk,
                     const float* v, int ldv, const float* o, int ldo, const float* lse,
                     const float* dout, int lddo, float* dq, int lddq, float* dk, int lddk,
                     float* dv, int lddv) {
    const int H = a->H, T = a->T, hd = a->hd;
    int kend_all = a->nvalid < a->Tk ? a->nvalid : a->Tk;
#pragma omp parallel for schedule(dynamic)
    for (int h = 0; h < H; ++h) {
        float* P = (float*)malloc(sizeof(float) * (size_t)T * (kend_all + 1));
        float* dS = (float*)malloc(sizeof(float) * (size_t)T * (kend_all + 1));
        for (int i = 0; i < T; ++i) {
            const float* qi = q + (size_t)i * ldq + h * hd;
            const float* oi = o + (size_t)i * ldo + h * hd;
            const float* doi = dout + (size_t)i * lddo + h * hd;
            int kend = kend_all;
            if (a->causal && kend > i + 1) kend = i + 1;
            float Di = 0;
            for (int c = 0; c < hd; ++c) Di += doi[c] * oi[c];
            for (int j = 0; j < kend_all; ++j) {
                float p = 0, ds = 0;
                if (j < kend) {
                    const float* kj = k + (size_t)j * ldk + h * hd;
                    const float* vj = v + (size_t)j * ldv + h * hd;
                    float d = 0, dp = 0;
                    for (int c = 0; c < hd; ++c) { d += qi[c] * kj[c]; dp += doi[c] * vj[c]; }
                    p = expf(d * a->scale - lse[(size_t)h * T + i]);
                    ds = p * (dp - Di);
                }
                P[(size_t)i * kend_all + j] = p;
                dS[(size_t)i * kend_all + j] = ds;
            }
            /* dq_i = scale * sum_j dS_ij k_j   (j ascending for every element) */
            float* dqi = dq + (size_t)i * lddq + h * hd;
            float acc[256];
            for (int c = 0; c < hd; ++c) acc[c] = 0;
            for (int j = 0; j < kend_all; ++j) {
                const float ds = dS[(size_t)i * kend_all + j];
                const float* kj = k + (size_t)j * ldk + h * hd;
                for (int c = 0; c < hd; ++c) acc[c] += ds * kj[c];
            }
            for (int c = 0; c < hd; ++c) dqi[c] = acc[c] * a->scale;
        }
        /* dk_j += scale * sum_i dS_ij q_i, dv_j += sum_i P_ij dO_i   (i ascending for every element) */
        float* ak = (float*)calloc((size_t)kend_all * hd + 1, sizeof(float));
        float* av = (float*)calloc((size_t)kend_all * hd + 1, sizeof(float));
        for (int i = 0; i < T; ++i) {
            const float* qi = q + (size_t)i * ldq + h * hd;
            const float* doi = dout + (size_t)i * lddo + h * hd;
            for (int j = 0; j < kend_all; ++j) {
                const float ds = dS[(size_t)i * kend_all + j], p = P[(size_t)i * kend_all + j];
                float* akj = ak + (size_t)j * hd;
                float* avj = av + (size_t)j * hd;
                for (int c = 0; c < hd; ++c) {
                    akj[c] += ds * qi[c];
                    avj[c] += p * doi[c];
                }
            }
        }
        for (int j = 0; j < kend_all; ++j) {
            float* dkj = dk + (size_t)j * lddk + h * hd;
            float* dvj = dv + (size_t)j * lddv + h * hd;
            for (int c = 0; c < hd; ++c) {
                dkj[c] += ak[(size_t)j * hd + c] * a->scale;
                dvj[c] += av[(size_t)j * hd + c];
            }
        }
        free(ak);
        free(av);
        free(P);
        free(dS);
    }
}

/* ggml GGML_ROPE_TYPE_NORMAL with freq_base 1: theta_i = pos / ff[i], pairs (2i, 2i+1). */
static void rope_apply(int T, int H, int hd, float* x, int ldx, const float* ff, int inverse) {
#pragma omp parallel for schedule(static) if (T > 16)
    for (int p = 0; p < T; ++p)
        for (int h = 0; h < H; ++h)
            for (int i = 0; i < hd / 2; ++i) {
                const float theta = (float)p / ff[i];
                const float c = cosf(theta), s = inverse ? -sinf(theta) : sinf(theta);
                float* e = x + (size_t)p * ldx + h * hd + 2 * i;
                const float x0 = e[0], x1 = e[1];
                e[0] = x0 * c - x1 * s;
                e[1] = x0 * s + x1 * c;
            }
}

/* ------------------------------------------------------------------------------------ */
/* LoRA / DoRA-rows linear (src/ac/lora.h:50-83)                                         */

typedef struct {
    int in, out, r, dora;
    float s;
    const float *W, *A, *B, *m;      /* W [out][in], A [r][in], B [out][r], m [out] */
    float *gA, *gB, *gm;             /* gradient accumulators (NULL when frozen) */
    float *P, *G, *Q, *nsq, *g;      /* DoRA: W A^T [out][r], A A^T [r][r], B G, nsq, m/sqrt(nsq) */
    float* dg;                       /* DoRA: sum over rows of dY * Y_lin, accumulated over clips */
} lora_t;

/* src/ac/lora.h:11-32: sum_i W[o,i]^2 accumulated in double from in*1e-12, cast to float. */
ORA_API void ora_row_norm_sq(const float* W, int out, int in, float* nsq) {
    for (int o = 0; o < out; ++o) {
        double s = in * 1e-12;
        for (int i = 0; i < in; ++i) s += (double)W[(size_t)o * in + i] * W[(size_t)o * in + i];
        nsq[o] = (float)s;
    }
}

static void lora_prepare(lora_t* L) {
    if (!L->r || !L->dora) return;
    const int out = L->out, in = L->in, r = L->r;
    L->P = zalloc((size_t)out * r);
    L->G = zalloc((size_t)r * r);
    L->Q = zalloc((size_t)out * r);
    L->nsq = zalloc(out);
    L->g = zalloc(out);
    L->dg = zalloc(out);
    mm_nt(out, r, in, L->W, in, L->A, in, L->P, r, 1.0f, 0);
    mm_nt(r, r, in, L->A, in, L->A, in, L->G, r, 1.0f, 0);
    mm_nn(out, r, r, L->B, r, L->G, r, L->Q, r, 1.0f, 0);
    float* base = zalloc(out);
    ora_row_norm_sq(L->W, out, in, base);
    for (int o = 0; o < out; ++o) {
        float t2 = 0, t3 = 0;
        for (int j = 0; j < r; ++j) {
            t2 += L->P[(size_t)o * r + j] * L->B[(size_t)o * r + j];
            t3 += L->B[(size_t)o * r + j] * L->Q[(size_t)o * r + j];
        }
        L->nsq[o] = base[o] + 2.0f * L->s * t2 + L->s * L->s * t3;
        L->g[o] = L->m[o] / sqrtf(L->nsq[o]);
    }
    free(base);
}

static void lora_release(lora_t* L) {
    free(L->P); free(L->G); free(L->Q); free(L->nsq); free(L->g); free(L->dg);
    L->P = L->G = L->Q = L->nsq = L->g = L->dg = NULL;
}

/* Y = (X W^T + s (X A^T) B^T) * g.  Saves U = X A^T and Y_lin (pre-DoRA) when given. */
static void lora_fwd(const lora_t* L, int n, const float* X, float* Y, float* U, float* Ylin) {
    mm_nt(n, L->out, L->in, X, L->in, L->W, L->in, Y, L->out, 1.0f, 0);
    if (!L->r) return;
    mm_nt(n, L->r, L->in, X, L->in, L->A, L->in, U, L->r, 1.0f, 0);
    mm_nt(n, L->out, L->r, U, L->r, L->B, L->r, Y, L->out, L->s, 1);
    if (L->dora) {
        memcpy(Ylin, Y, sizeof(float) * (size_t)n * L->out);
        for (int i = 0; i < n; ++i)
            for (int o = 0; o < L->out; ++o) Y[(size_t)i * L->out + o] *= L->g[o];
    }
}

/* dX (+)= grad of input; accumulates gA, gB (linear part) and dg (DoRA). dX may be NULL. */
static void lora_bwd(lora_t* L, int n, const float* X, const float* U, const float* Ylin,
                     const float* dY, float* dX, int accumulate_dx) {
    const int out = L->out, in = L->in, r = L->r;
    const float* dYl = dY;
    float* tmp = NULL;
    if (r && L->dora) {
        tmp = zalloc((size_t)n * out);
        for (int o = 0; o < out; ++o) {
            float acc = 0;
            for (int i = 0; i < n; ++i) acc += dY[(size_t)i * out + o] * Ylin[(size_t)i * out + o];
            L->dg[o] += acc;
        }
        for (int i = 0; i < n; ++i)
            for (int o = 0; o < out; ++o) tmp[(size_t)i * out + o] = dY[(size_t)i * out + o] * L->g[o];
        dYl = tmp;
    }
    if (dX) mm_nn(n, in, out, dYl, out, L->W, in, dX, in, 1.0f, accumulate_dx);
    if (r) {
        float* dU = zalloc((size_t)n * r);
        mm_nn(n, r, out, dYl, out, L->B, r, dU, r, L->s, 0);            /* dU = s dYl B */
        if (L->gB) mm_tn(out, r, n, dYl, out, U, r, L->gB, r, L->s, 1); /* dB += s dYl^T U */
        if (L->gA) mm_tn(r, in, n, dU, r, X, in, L->gA, in, 1.0f, 1);   /* dA += dU^T X */
        if (dX) mm_nn(n, in, r, dU, r, L->A, in, dX, in, 1.0f, 1);      /* dX += dU A */
        free(dU);
    }
    free(tmp);
}

/* After all rows: DoRA magnitude and norm terms (clip-independent part of the backward). */
static void lora_finish(lora_t* L) {
    if (!L->r || !L->dora) return;
    const int out = L->out, in = L->in, r = L->r;
    float* dt2 = zalloc(out);
    float* dt3 = zalloc(out);
    for (int o = 0; o < out; ++o) {
        const float sq = sqrtf(L->nsq[o]);
        if (L->gm) L->gm[o] += L->dg[o] / sq;
        const float dnsq = -0.5f * L->dg[o] * L->g[o] / L->nsq[o];
        dt2[o] = 2.0f * L->s * dnsq;
        dt3[o] = L->s * L->s * dnsq;
    }
    /* t2 = sum_j P[o,j] B[o,j]:  dB += dt2 * P ;  dA += (dt2 . B)^T W */
    /* t3 = B_o G B_o^T:          dB += 2 dt3 * Q ;  dA += 2 (B^T diag(dt3) B) A */
    if (L->gB)
        for (int o = 0; o < out; ++o)
            for (int j = 0; j < r; ++j)
                L->gB[(size_t)o * r + j] += dt2[o] * L->P[(size_t)o * r + j] +
                                            2.0f * dt3[o] * L->Q[(size_t)o * r + j];
    if (L->gA) {
        float* BD = zalloc((size_t)out * r); /* dt2[o] * B[o][j] */
        float* dG = zalloc((size_t)r * r);
        for (int o = 0; o < out; ++o)
            for (int j = 0; j < r; ++j) BD[(size_t)o * r + j] = dt2[o] * L->B[(size_t)o * r + j];
        mm_tn(r, in, out, BD, r, L->W, in, L->gA, in, 1.0f, 1);
        for (int o = 0; o < out; ++o)
            for (int j = 0; j < r; ++j)
                for (int k2 = 0; k2 < r; ++k2)
                    dG[(size_t)j * r + k2] += dt3[o] * L->B[(size_t)o * r + j] * L->B[(size_t)o * r + k2];
        mm_nn(r, in, r, dG, r, L->A, in, L->gA, in, 2.0f, 1);
        free(BD);
        free(dG);
    }
    free(dt2);
    free(dt3);
}

/* ------------------------------------------------------------------------------------ */
/* parameter / weight enumeration                                                         */

static const char* const TARGET_SUFFIX[7] = {"self.qkv", "self.out", "cross.q", "cross.kv",
                                              "cross.out", "ff.0", "ff.2"};

ORA_API const char* ora_target_suffix(int t) { return t >= 0 && t < 7 ? TARGET_SUFFIX[t] : ""; }

static void target_dims(int t, int D, int F, int* in, int* out) {
    static const int ins[7] = {1, 1, 1, 1, 1, 1, 0}, outs[7] = {3, 1, 1, 2, 1, 0, 1};
    *in = ins[t] ? D : F;
    *out = t == 5 ? F : outs[t] * D;
}

/* Number of floats the adapter parameters occupy, in the reference order:
 * for layer in [first_layer, L): for target in mask order: A [r][in], B [out][r], (m [out]). */
ORA_API int64_t ora_adapter_numel(int D, int F, int layers, const ora_adapter* ad) {
    int64_t n = 0;
    for (int l = ad->first_layer; l < layers; ++l)
        for (int t = 0; t < 7; ++t) {
            if (!(ad->targets >> t & 1)) continue;
            int in, out;
            target_dims(t, D, F, &in, &out);
            n += (int64_t)ad->rank * in + (int64_t)out * ad->rank + (ad->dora ? out : 0);
        }
    return n;
}

/* DiT base weights, flat fp32 in this fixed order (each [out][in] row-major):
 *  in_proj [D][lat], out_proj [lat][D], time_embed.0 [D][tdim], time_embed.2 [D][D],
 *  cond_proj.weight [D][cond], cond_proj.bias [D], rope_freq_factors [hd/2],
 *  out_norm.weight [D], out_norm.bias [D], skip.i [D][2D] (i < n_skip), then per layer:
 *  norm1.w, norm1.b, norm_cross.w, norm_cross.b, norm2.w, norm2.b, self.qkv, self.out,
 *  cross.q, cross.kv, cross.out, ff.0, ff.2. */
typedef struct {
    const float *in_proj, *out_proj, *te0, *te2, *cond_w, *cond_b, *ff, *onw, *onb;
    const float** skip;
    const float** layer; /* per layer 13 pointers */
    const float** all;   /* owns the pointer table */
} dit_weights;

ORA_API int ora_dit_tensor_count(const ora_dit_cfg* c) { return 9 + c->n_skip + 13 * c->layers; }

ORA_API int64_t ora_dit_tensor_shape(const ora_dit_cfg* c, int idx, int* rows, int* cols) {
    const int D = c->dim, F = c->ff_dim;
    int r = 1, k = 1;
    if (idx == 0) { r = D; k = c->latent_dim; }
    else if (idx == 1) { r = c->latent_dim; k = D; }
    else if (idx == 2) { r = D; k = c->time_dim; }
    else if (idx == 3) { r = D; k = D; }
    else if (idx == 4) { r = D; k = c->cond_dim; }
    else if (idx == 5 || idx == 7 || idx == 8) { r = 1; k = D; }
    else if (idx == 6) { r = 1; k = c->head_dim / 2; }
    else if (idx < 9 + c->n_skip) { r = D; k = 2 * D; }
    else {
        const int j = (idx - 9 - c->n_skip) % 13;
        if (j < 6) { r = 1; k = D; }
        else {
            int in, out;
            target_dims(j - 6, D, F, &in, &out);
            r = out;
            k = in;
        }
    }
    *rows = r;
    *cols = k;
    return (int64_t)r * k;
}

static void dit_map(const ora_dit_cfg* c, const float* W, dit_weights* w) {
    const float** ptr = (const float**)malloc(sizeof(float*) * ora_dit_tensor_count(c));
    int64_t off = 0;
    for (int i = 0; i < ora_dit_tensor_count(c); ++i) {
        int r, k;
        ptr[i] = W + off;
        off += ora_dit_tensor_shape(c, i, &r, &k);
    }
    w->in_proj = ptr[0]; w->out_proj = ptr[1]; w->te0 = ptr[2]; w->te2 = ptr[3];
    w->cond_w = ptr[4]; w->cond_b = ptr[5]; w->ff = ptr[6]; w->onw = ptr[7]; w->onb = ptr[8];
    w->skip = ptr + 9;
    w->layer = ptr + 9 + c->n_skip;
    w->all = ptr;
}

/* Build lora_t for every projection of every layer (r = 0 where not adapted). */
static lora_t* make_loras(int layers, int D, int F, const float** layer_w, const ora_adapter* ad,
                          const float* params, float* grads) {
    lora_t* Ls = (lora_t*)calloc((size_t)layers * 7, sizeof(lora_t));
    int64_t off = 0;
    for (int l = 0; l < layers; ++l)
        for (int t = 0; t < 7; ++t) {
            lora_t* L = &Ls[l * 7 + t];
            target_dims(t, D, F, &L->in, &L->out);
            L->W = layer_w[l * 13 + 6 + t];
            if (l < ad->first_layer || !(ad->targets >> t & 1)) continue;
            L->r = ad->rank;
            L->dora = ad->dora;
            L->s = ad->alpha / (float)ad->rank;
            L->A = params + off;
            if (grads) L->gA = grads + off;
            off += (int64_t)L->r * L->in;
            L->B = params + off;
            if (grads) L->gB = grads + off;
            off += (int64_t)L->out * L->r;
            if (L->dora) {
                L->m = params + off;
                if (grads) L->gm = grads + off;
                off += L->out;
            }
            lora_prepare(L);
        }
    return Ls;
}

static void free_loras(lora_t* Ls, int n) {
    for (int i = 0; i < n; ++i) lora_release(&Ls[i]);
    free(Ls);
}

/* ------------------------------------------------------------------------------------ */
/* one projection call site: input pointer plus what its backward needs                   */

typedef struct {
    float *Y, *U, *Ylin;
} proj_rec;

static void proj_run(lora_t* L, int n, const float* X, proj_rec* rec) {
    rec->Y = zalloc((size_t)n * L->out);
    rec->U = L->r ? zalloc((size_t)n * L->r) : NULL;
    rec->Ylin = L->r && L->dora ? zalloc((size_t)n * L->out) : NULL;
    lora_fwd(L, n, X, rec->Y, rec->U, rec->Ylin);
}

static void proj_free(proj_rec* r) {
    free(r->Y); free(r->U); free(r->Ylin);
    r->Y = r->U = r->Ylin = NULL;
}

/* ------------------------------------------------------------------------------------ */
/* MelodyFlow DiT step (src/mf/train.h:148-188 with dit_forward, src/mf/dit.h:160-212)     */

typedef struct {
    float *x_in, *mu1, *rs1, *h1;
    proj_rec qkv;  /* pre-RoPE projection output */
    float *qkv_rot, *o1, *lse1;
    proj_rec out;
    float *x_mid, *mu2, *rs2, *hc;
    proj_rec cq, ckv;
    float *o2, *lse2;
    proj_rec cout;
    float *x_mid2, *mu3, *rs3, *f;
    proj_rec f0;
    float* gact;
    proj_rec f2;
    float* x_out;
    float* skip_in; /* [T][2D] when the layer consumes a skip */
} dit_layer_act;

ORA_API int ora_dit_step(const ora_dit_cfg* c, const float* Wflat, const ora_adapter* ad,
                         const float* params, int n_clips, int T, int C, const float* clean,
                         const float* noise, const float* hidden, const float* tvals,
                         const int* uncond, const int* valid, float* loss_out, float* grads) {
    const int D = c->dim, F = c->ff_dim, H = c->heads, hd = c->head_dim, LAT = c->latent_dim;
    const int L = c->layers;
    if (D != H * hd || c->n_skip != (L - 1) / 2) return -1;
    if (ad->rank <= 0 || ad->first_layer < 0 || ad->first_layer >= L) return -2;
    dit_weights w;
    dit_map(c, Wflat, &w);
    lora_t* Ls = make_loras(L, D, F, w.layer, ad, params, grads);
    const float scale = 1.0f / sqrtf((float)hd);

    for (int b = 0; b < n_clips; ++b) {
        const float t = tvals[b];
        const float* cl = clean + (size_t)b * LAT * T;
        const float* nz = noise + (size_t)b * LAT * T;
        const float* hid = hidden + (size_t)b * C * c->cond_dim;
        /* --- inputs: x_t = (1-t) noise + t clean, v* = clean - noise (src/mf/train.h:156-159) */
        float* X0 = zalloc((size_t)T * LAT);
        float* vstar = zalloc((size_t)T * LAT);
        const float rescale = ora_dit_input_rescale(t);
        for (int ch = 0; ch < LAT; ++ch)
            for (int p = 0; p < T; ++p) {
                const size_t i = (size_t)ch * T + p;
                X0[(size_t)p * LAT + ch] = ((1 - t) * nz[i] + t * cl[i]) * rescale;
                vstar[i] = cl[i] - nz[i];
            }
        float* x = zalloc((size_t)T * D);
        mm_nt(T, D, LAT, X0, LAT, w.in_proj, LAT, x, D, 1.0f, 0);
        /* timestep embedding: W2 silu(W0 tfeat) */
        float* tfeat = zalloc(c->time_dim);
        ora_timestep_features(t, c->time_dim, 10000.0f, tfeat);
        float* te1 = zalloc(D);
        float* te = zalloc(D);
        mm_nt(1, D, c->time_dim, tfeat, c->time_dim, w.te0, c->time_dim, te1, D, 1.0f, 0);
        for (int j = 0; j < D; ++j) te1[j] = te1[j] / (1.0f + expf(-te1[j]));
        mm_nt(1, D, D, te1, D, w.te2, D, te, D, 1.0f, 0);
        /* projected conditioning */
        float* ctx = zalloc((size_t)C * D);
        mm_nt(C, D, c->cond_dim, hid, c->cond_dim, w.cond_w, c->cond_dim, ctx, D, 1.0f, 0);
        for (int i = 0; i < C; ++i)
            for (int j = 0; j < D; ++j) ctx[(size_t)i * D + j] += w.cond_b[j];
        const int nvalid = uncond[b] ? 0 : (valid && valid[b] >= 0 ? valid[b] : C);

        dit_layer_act* act = (dit_layer_act*)calloc(L, sizeof(dit_layer_act));
        int* stack = (int*)malloc(sizeof(int) * (L + 1));
        int* pair = (int*)malloc(sizeof(int) * L); /* producer popped by consumer l */
        int sp = 0;
        for (int l = 0; l < L; ++l) {
            dit_layer_act* a = &act[l];
            const float** lw = w.layer + l * 13;
            lora_t* Ll = Ls + l * 7;
            int cons, prod, proj;
            ora_skip_plan(l, L, c->n_skip, &cons, &prod, &proj);
            pair[l] = -1;
            if (cons) {
                const int src = stack[--sp];
                pair[l] = src;
                a->skip_in = zalloc((size_t)T * 2 * D);
                for (int p = 0; p < T; ++p) {
                    memcpy(a->skip_in + (size_t)p * 2 * D, x + (size_t)p * D, sizeof(float) * D);
                    memcpy(a->skip_in + (size_t)p * 2 * D + D, act[src].x_out + (size_t)p * D,
                           sizeof(float) * D);
                }
                mm_nt(T, D, 2 * D, a->skip_in, 2 * D, w.skip[proj], 2 * D, x, D, 1.0f, 0);
            }
            a->x_in = x;
            /* self-attention */
            a->mu1 = zalloc(T); a->rs1 = zalloc(T); a->h1 = zalloc((size_t)T * D);
            ln_fwd(T, D, a->x_in, lw[0], lw[1], c->norm_eps, te, a->h1, a->mu1, a->rs1);
            proj_run(&Ll[0], T, a->h1, &a->qkv);
            a->qkv_rot = zalloc((size_t)T * 3 * D);
            memcpy(a->qkv_rot, a->qkv.Y, sizeof(float) * (size_t)T * 3 * D);
            rope_apply(T, H, hd, a->qkv_rot, 3 * D, w.ff, 0);      /* q */
            rope_apply(T, H, hd, a->qkv_rot + D, 3 * D, w.ff, 0);  /* k */
            a->o1 = zalloc((size_t)T * D);
            a->lse1 = zalloc((size_t)H * T);
            attn_shape sa = {T, T, H, hd, c->add_zero_attn, 0, T, scale};
            attn_fwd(&sa, a->qkv_rot, 3 * D, a->qkv_rot + D, 3 * D, a->qkv_rot + 2 * D, 3 * D,
                     a->o1, D, a->lse1);
            proj_run(&Ll[1], T, a->o1, &a->out);
            a->x_mid = zalloc((size_t)T * D);
            for (size_t i = 0; i < (size_t)T * D; ++i) a->x_mid[i] = a->x_in[i] + a->out.Y[i];
            /* cross-attention */
            a->mu2 = zalloc(T); a->rs2 = zalloc(T); a->hc = zalloc((size_t)T * D);
            ln_fwd(T, D, a->x_mid, lw[2], lw[3], c->norm_eps, te, a->hc, a->mu2, a->rs2);
            proj_run(&Ll[2], T, a->hc, &a->cq);
            proj_run(&Ll[3], C, ctx, &a->ckv);
            a->o2 = zalloc((size_t)T * D);
            a->lse2 = zalloc((size_t)H * T);
            attn_shape ca = {T, C, H, hd, c->add_zero_attn, 0, nvalid, scale};
            attn_fwd(&ca, a->cq.Y, D, a->ckv.Y, 2 * D, a->ckv.Y + D, 2 * D, a->o2, D, a->lse2);
            proj_run(&Ll[4], T, a->o2, &a->cout);
            a->x_mid2 = zalloc((size_t)T * D);
            for (size_t i = 0; i < (size_t)T * D; ++i) a->x_mid2[i] = a->x_mid[i] + a->cout.Y[i];
            /* feed-forward (no timestep) */
            a->mu3 = zalloc(T); a->rs3 = zalloc(T); a->f = zalloc((size_t)T * D);
            ln_fwd(T, D, a->x_mid2, lw[4], lw[5], c->norm_eps, NULL, a->f, a->mu3, a->rs3);
            proj_run(&Ll[5], T, a->f, &a->f0);
            a->gact = zalloc((size_t)T * F);
            for (size_t i = 0; i < (size_t)T * F; ++i) a->gact[i] = ora_gelu(a->f0.Y[i]);
            proj_run(&Ll[6], T, a->gact, &a->f2);
            a->x_out = zalloc((size_t)T * D);
            for (size_t i = 0; i < (size_t)T * D; ++i) a->x_out[i] = a->x_mid2[i] + a->f2.Y[i];
            x = zalloc((size_t)T * D);
            memcpy(x, a->x_out, sizeof(float) * (size_t)T * D);
            if (prod) stack[sp++] = l;
        }
        /* output head: LN -> out_proj -> transpose -> * sqrt(2); MSE (src/mf/train.h:107) */
        float *muo = zalloc(T), *rso = zalloc(T), *xo = zalloc((size_t)T * D);
        ln_fwd(T, D, x, w.onw, w.onb, c->norm_eps, NULL, xo, muo, rso);
        float* outp = zalloc((size_t)T * LAT);
        mm_nt(T, LAT, D, xo, D, w.out_proj, D, outp, LAT, 1.0f, 0);
        const float sq2 = sqrtf(2.0f);
        float loss = 0;
        float* dout = zalloc((size_t)T * LAT);
        const float inv = 1.0f / (float)(T * LAT);
        for (int ch = 0; ch < LAT; ++ch)
            for (int p = 0; p < T; ++p) {
                const float v = outp[(size_t)p * LAT + ch] * sq2;
                const float d = v - vstar[(size_t)ch * T + p];
                loss += d * d;
                dout[(size_t)p * LAT + ch] = 2.0f * d * inv * sq2;
            }
        loss_out[b] = loss * inv;

        if (grads) {
            /* ---------------------------- backward ---------------------------- */
            float* dxo = zalloc((size_t)T * D);
            mm_nn(T, D, LAT, dout, LAT, w.out_proj, D, dxo, D, 1.0f, 0);
            float* dx = zalloc((size_t)T * D);
            ln_bwd(T, D, x, w.onw, muo, rso, dxo, dx);
            free(dxo);
            float** dsaved = (float**)calloc(L, sizeof(float*));
            for (int l = L - 1; l >= ad->first_layer; --l) {
                dit_layer_act* a = &act[l];
                const float** lw = w.layer + l * 13;
                lora_t* Ll = Ls + l * 7;
                if (dsaved[l]) {
                    for (size_t i = 0; i < (size_t)T * D; ++i) dx[i] += dsaved[l][i];
                    free(dsaved[l]);
                    dsaved[l] = NULL;
                }
                /* feed-forward */
                float* dg = zalloc((size_t)T * F);
                lora_bwd(&Ll[6], T, a->gact, a->f2.U, a->f2.Ylin, dx, dg, 0);
                for (size_t i = 0; i < (size_t)T * F; ++i) dg[i] *= ora_gelu_grad(a->f0.Y[i]);
                float* df = zalloc((size_t)T * D);
                lora_bwd(&Ll[5], T, a->f, a->f0.U, a->f0.Ylin, dg, df, 0);
                free(dg);
                ln_bwd(T, D, a->x_mid2, lw[4], a->mu3, a->rs3, df, dx);
                free(df);
                /* cross-attention */
                float* do2 = zalloc((size_t)T * D);
                lora_bwd(&Ll[4], T, a->o2, a->cout.U, a->cout.Ylin, dx, do2, 0);
                float* dcq = zalloc((size_t)T * D);
                float* dckv = zalloc((size_t)C * 2 * D);
                attn_shape ca = {T, C, H, hd, c->add_zero_attn, 0, nvalid, scale};
                attn_bwd(&ca, a->cq.Y, D, a->ckv.Y, 2 * D, a->ckv.Y + D, 2 * D, a->o2, D, a->lse2,
                         do2, D, dcq, D, dckv, 2 * D, dckv + D, 2 * D);
                free(do2);
                lora_bwd(&Ll[3], C, ctx, a->ckv.U, a->ckv.Ylin, dckv, NULL, 0);
                free(dckv);
                float* dhc = zalloc((size_t)T * D);
                lora_bwd(&Ll[2], T, a->hc, a->cq.U, a->cq.Ylin, dcq, dhc, 0);
                free(dcq);
                ln_bwd(T, D, a->x_mid, lw[2], a->mu2, a->rs2, dhc, dx);
                free(dhc);
                /* self-attention */
                float* do1 = zalloc((size_t)T * D);
                lora_bwd(&Ll[1], T, a->o1, a->out.U, a->out.Ylin, dx, do1, 0);
                float* dqkv = zalloc((size_t)T * 3 * D);
                attn_shape sa = {T, T, H, hd, c->add_zero_attn, 0, T, scale};
                attn_bwd(&sa, a->qkv_rot, 3 * D, a->qkv_rot + D, 3 * D, a->qkv_rot + 2 * D, 3 * D,
                         a->o1, D, a->lse1, do1, D, dqkv, 3 * D, dqkv + D, 3 * D, dqkv + 2 * D, 3 * D);
                free(do1);
                rope_apply(T, H, hd, dqkv, 3 * D, w.ff, 1);
                rope_apply(T, H, hd, dqkv + D, 3 * D, w.ff, 1);
                float* dh = zalloc((size_t)T * D);
                lora_bwd(&Ll[0], T, a->h1, a->qkv.U, a->qkv.Ylin, dqkv, dh, 0);
                free(dqkv);
                ln_bwd(T, D, a->x_in, lw[0], a->mu1, a->rs1, dh, dx);
                free(dh);
                /* skip projection: x_new = Wskip [x; saved] */
                if (a->skip_in) {
                    int cons, prod, proj;
                    ora_skip_plan(l, L, c->n_skip, &cons, &prod, &proj);
                    float* dcat = zalloc((size_t)T * 2 * D);
                    mm_nn(T, 2 * D, D, dx, D, w.skip[proj], 2 * D, dcat, 2 * D, 1.0f, 0);
                    const int src = pair[l];
                    if (!dsaved[src]) dsaved[src] = zalloc((size_t)T * D);
                    for (int p = 0; p < T; ++p)
                        for (int j = 0; j < D; ++j) {
                            dx[(size_t)p * D + j] = dcat[(size_t)p * 2 * D + j];
                            dsaved[src][(size_t)p * D + j] += dcat[(size_t)p * 2 * D + D + j];
                        }
                    free(dcat);
                }
            }
            for (int l = 0; l < L; ++l) free(dsaved[l]);
            free(dsaved);
            free(dx);
        }
        /* release per-clip storage */
        for (int l = 0; l < L; ++l) {
            dit_layer_act* a = &act[l];
            free(a->x_in); free(a->mu1); free(a->rs1); free(a->h1); proj_free(&a->qkv);
            free(a->qkv_rot); free(a->o1); free(a->lse1); proj_free(&a->out); free(a->x_mid);
            free(a->mu2); free(a->rs2); free(a->hc); proj_free(&a->cq); proj_free(&a->ckv);
            free(a->o2); free(a->lse2); proj_free(&a->cout); free(a->x_mid2); free(a->mu3);
            free(a->rs3); free(a->f); proj_free(&a->f0); free(a->gact); proj_free(&a->f2);
            free(a->x_out); free(a->skip_in);
        }
        free(act); free(stack); free(pair); free(x);
        free(X0); free(vstar); free(tfeat); free(te1); free(te); free(ctx);
        free(muo); free(rso); free(xo); free(outp); free(dout);
    }
    if (grads)
        for (int i = 0; i < L * 7; ++i) lora_finish(&Ls[i]);
    free_loras(Ls, L * 7);
    free((void*)w.all);
    return 0;
}

/* ------------------------------------------------------------------------------------ */
/* MusicGen LM step (src/mg/train.h:12-49,131,178-227)                                    */

/* LM weights, flat fp32, fixed order: emb.q [card+1][D] (q < n_q), head.q [card][D],
 * out_norm.w, out_norm.b, then per layer the same 13 tensors as the DiT. */
ORA_API int ora_lm_tensor_count(const ora_lm_cfg* c) { return 2 * c->n_q + 2 + 13 * c->layers; }

ORA_API int64_t ora_lm_tensor_shape(const ora_lm_cfg* c, int idx, int* rows, int* cols) {
    const int D = c->dim, F = c->ff_dim;
    int r = 1, k = 1;
    if (idx < c->n_q) { r = c->card + 1; k = D; }
    else if (idx < 2 * c->n_q) { r = c->card; k = D; }
    else if (idx < 2 * c->n_q + 2) { r = 1; k = D; }
    else {
        const int j = (idx - 2 * c->n_q - 2) % 13;
        if (j < 6) { r = 1; k = D; }
        else {
            int in, out;
            target_dims(j - 6, D, F, &in, &out);
            r = out;
            k = in;
        }
    }
    *rows = r;
    *cols = k;
    return (int64_t)r * k;
}

typedef struct {
    float *x_in, *mu1, *rs1, *h1;
    proj_rec qkv;
    float *o1, *lse1;
    proj_rec out;
    float *x_mid, *mu2, *rs2, *hc;
    proj_rec cq, ckv;
    float *o2, *lse2;
    proj_rec cout;
    float *x_mid2, *mu3, *rs3, *f;
    proj_rec f0;
    float* gact;
    proj_rec f2;
} lm_layer_act;

/* codes [n][n_q][frames]; context [n][C][D] (already projected); loss_out [n]. */
ORA_API int ora_lm_step(const ora_lm_cfg* c, const float* Wflat, const ora_adapter* ad,
                        const float* params, int n_seq, int frames, int prefix, int C,
                        const int32_t* codes, const float* context, float* loss_out,
                        float* grads) {
    const int D = c->dim, F = c->ff_dim, H = c->heads, hd = c->head_dim, L = c->layers;
    const int NQ = c->n_q, CARD = c->card;
    if (D != H * hd || prefix < 0 || prefix >= frames) return -1;
    const int S = 1 + frames + (NQ - 1); /* pattern steps */
    const int steps = S - 1;             /* src/mg/train.h:74 */
    const float** ptr = (const float**)malloc(sizeof(float*) * ora_lm_tensor_count(c));
    int64_t off = 0;
    for (int i = 0; i < ora_lm_tensor_count(c); ++i) {
        int r, k;
        ptr[i] = Wflat + off;
        off += ora_lm_tensor_shape(c, i, &r, &k);
    }
    const float** emb = ptr;
    const float** head = ptr + NQ;
    const float *onw = ptr[2 * NQ], *onb = ptr[2 * NQ + 1];
    const float** layer_w = ptr + 2 * NQ + 2;
    lora_t* Ls = make_loras(L, D, F, layer_w, ad, params, grads);
    const float scale = 1.0f / sqrtf((float)hd);
    float* pos = zalloc((size_t)steps * D);
    ora_sin_positions(0, steps, D, c->pos_denominator, c->max_period, pos);

    for (int b = 0; b < n_seq; ++b) {
        const int32_t* cd = codes + (size_t)b * NQ * frames;
        const float* ctx = context + (size_t)b * C * D;
        int32_t* seq = (int32_t*)malloc(sizeof(int32_t) * (size_t)NQ * S);
        ora_pattern_build(NQ, frames, cd, c->special_token_id, seq);
        float* x = zalloc((size_t)steps * D);
        for (int s = 0; s < steps; ++s) {
            for (int q = 0; q < NQ; ++q) {
                const int id = seq[(size_t)q * S + s];
                for (int j = 0; j < D; ++j) x[(size_t)s * D + j] += emb[q][(size_t)id * D + j];
            }
            for (int j = 0; j < D; ++j) x[(size_t)s * D + j] += pos[(size_t)s * D + j];
        }
        lm_layer_act* act = (lm_layer_act*)calloc(L, sizeof(lm_layer_act));
        for (int l = 0; l < L; ++l) {
            lm_layer_act* a = &act[l];
            const float** lw = layer_w + l * 13;
            lora_t* Ll = Ls + l * 7;
            a->x_in = x;
            a->mu1 = zalloc(steps); a->rs1 = zalloc(steps); a->h1 = zalloc((size_t)steps * D);
            ln_fwd(steps, D, x, lw[0], lw[1], c->norm_eps, NULL, a->h1, a->mu1, a->rs1);
            proj_run(&Ll[0], steps, a->h1, &a->qkv);
            a->o1 = zalloc((size_t)steps * D);
            a->lse1 = zalloc((size_t)H * steps);
            attn_shape sa = {steps, steps, H, hd, 0, 1, steps, scale};
            attn_fwd(&sa, a->qkv.Y, 3 * D, a->qkv.Y + D, 3 * D, a->qkv.Y + 2 * D, 3 * D, a->o1, D,
                     a->lse1);
            proj_run(&Ll[1], steps, a->o1, &a->out);
            a->x_mid = zalloc((size_t)steps * D);
            for (size_t i = 0; i < (size_t)steps * D; ++i) a->x_mid[i] = a->x_in[i] + a->out.Y[i];
            a->mu2 = zalloc(steps); a->rs2 = zalloc(steps); a->hc = zalloc((size_t)steps * D);
            ln_fwd(steps, D, a->x_mid, lw[2], lw[3], c->norm_eps, NULL, a->hc, a->mu2, a->rs2);
            proj_run(&Ll[2], steps, a->hc, &a->cq);
            proj_run(&Ll[3], C, ctx, &a->ckv);
            a->o2 = zalloc((size_t)steps * D);
            a->lse2 = zalloc((size_t)H * steps);
            attn_shape ca = {steps, C, H, hd, 0, 0, C, scale};
            attn_fwd(&ca, a->cq.Y, D, a->ckv.Y, 2 * D, a->ckv.Y + D, 2 * D, a->o2, D, a->lse2);
            proj_run(&Ll[4], steps, a->o2, &a->cout);
            a->x_mid2 = zalloc((size_t)steps * D);
            for (size_t i = 0; i < (size_t)steps * D; ++i) a->x_mid2[i] = a->x_mid[i] + a->cout.Y[i];
            a->mu3 = zalloc(steps); a->rs3 = zalloc(steps); a->f = zalloc((size_t)steps * D);
            ln_fwd(steps, D, a->x_mid2, lw[4], lw[5], c->norm_eps, NULL, a->f, a->mu3, a->rs3);
            proj_run(&Ll[5], steps, a->f, &a->f0);
            a->gact = zalloc((size_t)steps * F);
            for (size_t i = 0; i < (size_t)steps * F; ++i) a->gact[i] = ora_gelu(a->f0.Y[i]);
            proj_run(&Ll[6], steps, a->gact, &a->f2);
            x = zalloc((size_t)steps * D);
            for (size_t i = 0; i < (size_t)steps * D; ++i) x[i] = a->x_mid2[i] + a->f2.Y[i];
        }
        float *muo = zalloc(steps), *rso = zalloc(steps), *xo = zalloc((size_t)steps * D);
        ln_fwd(steps, D, x, onw, onb, c->norm_eps, NULL, xo, muo, rso);
        /* selected rows: (q, s) with timestep_at(q, s+1) >= prefix (src/mg/train.h:192-199) */
        const int nsel = NQ * (frames - prefix);
        float* dxo = grads ? zalloc((size_t)steps * D) : NULL;
        double loss = 0;
        float* logit = zalloc((size_t)steps * CARD);
        float* dlogit = zalloc((size_t)steps * CARD);
        for (int q = 0; q < NQ; ++q) {
            mm_nt(steps, CARD, D, xo, D, head[q], D, logit, CARD, 1.0f, 0);
            memset(dlogit, 0, sizeof(float) * (size_t)steps * CARD);
            for (int s = 0; s < steps; ++s) {
                const int t = pattern_timestep(q, s + 1, frames);
                if (t < prefix) continue;
                const int target = cd[(size_t)q * frames + t];
                const float* lg = logit + (size_t)s * CARD;
                float m = -INFINITY;
                for (int j = 0; j < CARD; ++j) m = lg[j] > m ? lg[j] : m;
                float sum = 0;
                for (int j = 0; j < CARD; ++j) sum += expf(lg[j] - m);
                loss += -(double)(lg[target] - m - logf(sum));
                for (int j = 0; j < CARD; ++j)
                    dlogit[(size_t)s * CARD + j] =
                        (expf(lg[j] - m) / sum - (j == target ? 1.0f : 0.0f)) / (float)nsel;
            }
            if (dxo) mm_nn(steps, D, CARD, dlogit, CARD, head[q], D, dxo, D, 1.0f, 1);
        }
        free(logit);
        free(dlogit);
        loss_out[b] = (float)(loss / nsel);
        if (grads) {
            float* dx = zalloc((size_t)steps * D);
            ln_bwd(steps, D, x, onw, muo, rso, dxo, dx);
            for (int l = L - 1; l >= ad->first_layer; --l) {
                lm_layer_act* a = &act[l];
                const float** lw = layer_w + l * 13;
                lora_t* Ll = Ls + l * 7;
                float* dg = zalloc((size_t)steps * F);
                lora_bwd(&Ll[6], steps, a->gact, a->f2.U, a->f2.Ylin, dx, dg, 0);
                for (size_t i = 0; i < (size_t)steps * F; ++i) dg[i] *= ora_gelu_grad(a->f0.Y[i]);
                float* df = zalloc((size_t)steps * D);
                lora_bwd(&Ll[5], steps, a->f, a->f0.U, a->f0.Ylin, dg, df, 0);
                free(dg);
                ln_bwd(steps, D, a->x_mid2, lw[4], a->mu3, a->rs3, df, dx);
                free(df);
                float* do2 = zalloc((size_t)steps * D);
                lora_bwd(&Ll[4], steps, a->o2, a->cout.U, a->cout.Ylin, dx, do2, 0);
                float* dcq = zalloc((size_t)steps * D);
                float* dckv = zalloc((size_t)C * 2 * D);
                attn_shape ca = {steps, C, H, hd, 0, 0, C, scale};
                attn_bwd(&ca, a->cq.Y, D, a->ckv.Y, 2 * D, a->ckv.Y + D, 2 * D, a->o2, D, a->lse2,
                         do2, D, dcq, D, dckv, 2 * D, dckv + D, 2 * D);
                free(do2);
                lora_bwd(&Ll[3], C, ctx, a->ckv.U, a->ckv.Ylin, dckv, NULL, 0);
                free(dckv);
                float* dhc = zalloc((size_t)steps * D);
                lora_bwd(&Ll[2], steps, a->hc, a->cq.U, a->cq.Ylin, dcq, dhc, 0);
                free(dcq);
                ln_bwd(steps, D, a->x_mid, lw[2], a->mu2, a->rs2, dhc, dx);
                free(dhc);
                float* do1 = zalloc((size_t)steps * D);
                lora_bwd(&Ll[1], steps, a->o1, a->out.U, a->out.Ylin, dx, do1, 0);
                float* dqkv = zalloc((size_t)steps * 3 * D);
                attn_shape sa = {steps, steps, H, hd, 0, 1, steps, scale};
                attn_bwd(&sa, a->qkv.Y, 3 * D, a->qkv.Y + D, 3 * D, a->qkv.Y + 2 * D, 3 * D, a->o1, D,
                         a->lse1, do1, D, dqkv, 3 * D, dqkv + D, 3 * D, dqkv + 2 * D, 3 * D);
                free(do1);
                float* dh = zalloc((size_t)steps * D);
                lora_bwd(&Ll[0], steps, a->h1, a->qkv.U, a->qkv.Ylin, dqkv, dh, 0);
                free(dqkv);
                ln_bwd(steps, D, a->x_in, lw[0], a->mu1, a->rs1, dh, dx);
                free(dh);
            }
            free(dx);
        }
        for (int l = 0; l < L; ++l) {
            lm_layer_act* a = &act[l];
            free(a->x_in); free(a->mu1); free(a->rs1); free(a->h1); proj_free(&a->qkv);
            free(a->o1); free(a->lse1); proj_free(&a->out); free(a->x_mid); free(a->mu2);
            free(a->rs2); free(a->hc); proj_free(&a->cq); proj_free(&a->ckv); free(a->o2);
            free(a->lse2); proj_free(&a->cout); free(a->x_mid2); free(a->mu3); free(a->rs3);
            free(a->f); proj_free(&a->f0); free(a->gact); proj_free(&a->f2);
        }
        free(act); free(x); free(muo); free(rso); free(xo); free(dxo); free(seq);
    }
    if (grads)
        for (int i = 0; i < L * 7; ++i) lora_finish(&Ls[i]);
    free_loras(Ls, L * 7);
    free(pos);
    free((void*)ptr);
    return 0;
}

/* ------------------------------------------------------------------------------------ */
/* optimizer                                                                              */

/* TrainControls::rate, src/ac/train_controls.h:53-58 */
ORA_API float ora_rate(float lr, int step, int warmup, int inverse) {
    float factor = warmup ? fminf(1.f, (float)step / (float)warmup) : 1.f;
    if (inverse) factor *= powf(1.f + (float)(step - 1) / 1000000.f, -.5f);
    return lr * factor;
}

/* TrainAccumulation::update, src/ac/train_controls.h:89-118.  grad holds the SUM over
 * `count` microbatches; decay[i] != 0 marks lora_A / lora_B entries.  Returns the number
 * of nonfinite updated values. */
ORA_API int64_t ora_adamw(int64_t n, float* value, float* m, float* v, float* grad,
                          const uint8_t* decays, int count, int step, float lr, float beta1,
                          float beta2, float eps, float decay, float clip) {
    double norm = 0;
    for (int64_t i = 0; i < n; ++i) {
        grad[i] /= (float)count;
        norm += (double)grad[i] * grad[i];
    }
    const float scale = (float)fmin(1., (double)clip / (sqrt(norm) + 1e-12));
    const float bc1 = 1 - powf(beta1, (float)step), bc2 = 1 - powf(beta2, (float)step);
    int64_t bad = 0;
    for (int64_t i = 0; i < n; ++i) {
        const float wd = decays[i] ? decay : 0.0f;
        const float g = scale * grad[i];
        m[i] = beta1 * m[i] + (1 - beta1) * g;
        v[i] = beta2 * v[i] + (1 - beta2) * g * g;
        value[i] -= lr * ((m[i] / bc1) / (sqrtf(v[i] / bc2) + eps) + wd * value[i]);
        if (!isfinite(value[i])) ++bad;
    }
    return bad;
}
