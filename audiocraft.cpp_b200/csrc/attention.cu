// attention.cu -- flash-style attention forward/backward for head_dim 64.
//
// Restates the training attention of src/ac/transformer.h:108-125 (dense softmax(scale K^T Q
// + mask) V with an optional prepended zero key, src/ac/transformer.h:74-79) without ever
// materialising the probabilities:
//   * the zero key is implicit: it starts the running max at 0 and the running sum at 1
//     (score 0, value 0), so it only enters through the log-sum-exp;
//   * masks are per-clip valid-key counts (the reference's -inf columns beyond
//     valid_tokens, src/mf/train.h:169-175) and an optional causal mask (src/mg/train.h:209-213);
//   * RoPE with stored frequencies (src/ac/transformer.h:55-61) is applied while Q and K
//     tiles are staged into shared memory, and undone in the dQ/dK epilogues.
// Backward follows the standard recompute scheme: P from the saved LSE, D = rowsum(dO*O),
// dS = P (dP - D); dK and dV are owned by key blocks, dQ accumulates through fp32 atomics.
#include "common.cuh"
#include "kernels.h"

#include <stdexcept>

namespace act {

namespace {

constexpr int HD = 64;
constexpr int BQ = 64;
constexpr int BKV = 64;
constexpr int LDS = HD + 8;
constexpr float LOG2E = 1.4426950408889634f;

// Stage a [64 rows][64] bf16 tile into smem, rotating pairs when rope != nullptr.
// Rows >= nrows are zero-filled.  pos0 is the clip position of row 0.
__device__ __forceinline__ void stage_tile(bf16* sm, const bf16* g, long ld, int nrows, int pos0,
                                           const float* rope, int tid, int nthreads) {
    for (int c = tid; c < 64 * 8; c += nthreads) {
        const int r = c >> 3, ch = c & 7;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < nrows) {
            v = *reinterpret_cast<const uint4*>(g + (long)r * ld + ch * 8);
            if (rope) {
                const float2* cs = reinterpret_cast<const float2*>(rope) + (long)(pos0 + r) * 32 + ch * 4;
                uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    __nv_bfloat162 b2 = *reinterpret_cast<__nv_bfloat162*>(&w[j]);
                    const float x0 = __low2float(b2), x1 = __high2float(b2);
                    const float2 t = cs[j];
                    w[j] = pack_bf16(x0 * t.x - x1 * t.y, x0 * t.y + x1 * t.x);
                }
            }
        }
        *reinterpret_cast<uint4*>(sm + r * LDS + ch * 8) = v;
    }
}

__global__ void __launch_bounds__(128) attn_fwd_kernel(const AttnArgs a) {
    __shared__ __align__(16) bf16 sQ[BQ * LDS];
    __shared__ __align__(16) bf16 sK[BKV * LDS];
    __shared__ __align__(16) bf16 sV[BKV * LDS];
    const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, q = lane & 3, lr = lane & 7, lsel = lane >> 3;
    const int q0 = qb * BQ;
    const int nq = min(BQ, a.T - q0);
    int kv_end = a.Tk;
    if (a.nvalid) kv_end = min(kv_end, a.nvalid[b]);
    if (a.causal) kv_end = min(kv_end, q0 + BQ);

    stage_tile(sQ, a.q + ((long)b * a.T + q0) * a.ldq + h * HD, a.ldq, nq, q0, a.rope, tid, 128);
    __syncthreads();
    uint32_t qf[4][4];
#pragma unroll
    for (int kc = 0; kc < 4; ++kc)
        ldsm_x4(qf[kc][0], qf[kc][1], qf[kc][2], qf[kc][3],
                sQ + (warp * 16 + lr + 8 * (lsel & 1)) * LDS + kc * 16 + 8 * (lsel >> 1));

    const float sl2 = a.scale * LOG2E;
    float mrow[2], lrow[2];
    mrow[0] = mrow[1] = a.zero_key ? 0.f : -INFINITY;
    lrow[0] = lrow[1] = a.zero_key ? 1.f : 0.f;
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[i][e] = 0.f;

    const int nkb = (kv_end + BKV - 1) / BKV;
    for (int kb = 0; kb < nkb; ++kb) {
        const int k0 = kb * BKV;
        __syncthreads();
        stage_tile(sK, a.k + ((long)b * a.Tk + k0) * a.ldk + h * HD, a.ldk, min(BKV, kv_end - k0), k0,
                   a.rope, tid, 128);
        stage_tile(sV, a.v + ((long)b * a.Tk + k0) * a.ldv + h * HD, a.ldv, min(BKV, kv_end - k0), k0,
                   nullptr, tid, 128);
        __syncthreads();
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) s[i][e] = 0.f;
#pragma unroll
        for (int kc = 0; kc < 4; ++kc)
#pragma unroll
            for (int nj = 0; nj < 4; ++nj) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(b0, b1, b2, b3, sK + (nj * 16 + lr + 8 * (lsel >> 1)) * LDS + kc * 16 + 8 * (lsel & 1));
                mma_bf16(s[2 * nj], qf[kc], b0, b1);
                mma_bf16(s[2 * nj + 1], qf[kc], b2, b3);
            }
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int ni = 0; ni < 8; ++ni)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = k0 + ni * 8 + 2 * q + (e & 1);
                const int i = q0 + warp * 16 + g + 8 * (e >> 1);
                const bool ok = j < kv_end && (!a.causal || j <= i);
                s[ni][e] = ok ? s[ni][e] * sl2 : -INFINITY;
                mx[e >> 1] = fmaxf(mx[e >> 1], s[ni][e]);
            }
        float alpha[2], muse[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 1));
            mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 2));
            const float mnew = fmaxf(mrow[hh], mx[hh]);
            muse[hh] = mnew == -INFINITY ? 0.f : mnew;
            alpha[hh] = exp2f(mrow[hh] - muse[hh]);
            mrow[hh] = mnew;
        }
        float rs[2] = {0.f, 0.f};
#pragma unroll
        for (int ni = 0; ni < 8; ++ni)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                s[ni][e] = exp2f(s[ni][e] - muse[e >> 1]);
                rs[e >> 1] += s[ni][e];
            }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            rs[hh] += __shfl_xor_sync(0xffffffffu, rs[hh], 1);
            rs[hh] += __shfl_xor_sync(0xffffffffu, rs[hh], 2);
            lrow[hh] = lrow[hh] * alpha[hh] + rs[hh];
        }
#pragma unroll
        for (int ni = 0; ni < 8; ++ni) {
            o[ni][0] *= alpha[0];
            o[ni][1] *= alpha[0];
            o[ni][2] *= alpha[1];
            o[ni][3] *= alpha[1];
        }
#pragma unroll
        for (int kc = 0; kc < 4; ++kc) {
            uint32_t pa[4];
            pa[0] = pack_bf16(s[2 * kc][0], s[2 * kc][1]);
            pa[1] = pack_bf16(s[2 * kc][2], s[2 * kc][3]);
            pa[2] = pack_bf16(s[2 * kc + 1][0], s[2 * kc + 1][1]);
            pa[3] = pack_bf16(s[2 * kc + 1][2], s[2 * kc + 1][3]);
#pragma unroll
            for (int nj = 0; nj < 4; ++nj) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(b0, b1, b2, b3, sV + (kc * 16 + lr + 8 * (lsel & 1)) * LDS + nj * 16 + 8 * (lsel >> 1));
                mma_bf16(o[2 * nj], pa, b0, b1);
                mma_bf16(o[2 * nj + 1], pa, b2, b3);
            }
        }
    }
    // epilogue
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int i = q0 + warp * 16 + g + 8 * hh;
        if (i >= a.T) continue;
        const float inv = lrow[hh] > 0.f ? 1.f / lrow[hh] : 0.f;
        bf16* orow = a.o + ((long)b * a.T + i) * a.ldo + h * HD;
#pragma unroll
        for (int ni = 0; ni < 8; ++ni)
            *reinterpret_cast<uint32_t*>(orow + ni * 8 + 2 * q) =
                pack_bf16(o[ni][2 * hh] * inv, o[ni][2 * hh + 1] * inv);
        if (q == 0) {
            const float mfin = mrow[hh] == -INFINITY ? 0.f : mrow[hh];
            a.lse[((long)b * a.H + h) * a.T + i] = mfin + log2f(lrow[hh]);
        }
    }
}

// D[b][h][i] = sum_d dO * O   (one warp per (row, head))
__global__ void attn_dvec_kernel(const AttnArgs a) {
    const long w = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    const long rows = (long)a.clips * a.T;
    if (w >= rows * a.H) return;
    const long row = w / a.H;
    const int h = (int)(w % a.H);
    const bf16* o = a.o + row * a.ldo + h * HD + 2 * lane;
    const bf16* d = a.dout + row * a.lddo + h * HD + 2 * lane;
    const __nv_bfloat162 o2 = *reinterpret_cast<const __nv_bfloat162*>(o);
    const __nv_bfloat162 d2 = *reinterpret_cast<const __nv_bfloat162*>(d);
    float v = __low2float(o2) * __low2float(d2) + __high2float(o2) * __high2float(d2);
    v = warp_sum(v);
    if (lane == 0) {
        const int b = (int)(row / a.T), i = (int)(row % a.T);
        a.dvec[((long)b * a.H + h) * a.T + i] = v;
    }
}

__global__ void __launch_bounds__(128) attn_bwd_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) unsigned char smraw[];
    bf16* sK = reinterpret_cast<bf16*>(smraw);
    bf16* sV = sK + BKV * LDS;
    bf16* sQ = sV + BKV * LDS;
    bf16* sdO = sQ + BQ * LDS;
    bf16* sP = sdO + BQ * LDS;
    bf16* sdS = sP + BQ * LDS;
    const int kb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, q = lane & 3, lr = lane & 7, lsel = lane >> 3;
    const int k0 = kb * BKV;
    int kv_end = a.Tk;
    if (a.nvalid) kv_end = min(kv_end, a.nvalid[b]);
    const int nk = max(0, min(BKV, kv_end - k0));

    stage_tile(sK, a.k + ((long)b * a.Tk + k0) * a.ldk + h * HD, a.ldk, nk, k0, a.rope, tid, 128);
    stage_tile(sV, a.v + ((long)b * a.Tk + k0) * a.ldv + h * HD, a.ldv, nk, k0, nullptr, tid, 128);

    const float sl2 = a.scale * LOG2E;
    float dk[8][4], dv[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

    const int qb0 = a.causal ? k0 / BQ : 0;
    const int nqb = (a.T + BQ - 1) / BQ;
    for (int qb = (nk > 0 ? qb0 : nqb); qb < nqb; ++qb) {
        const int q0 = qb * BQ;
        const int nq = min(BQ, a.T - q0);
        __syncthreads();
        stage_tile(sQ, a.q + ((long)b * a.T + q0) * a.ldq + h * HD, a.ldq, nq, q0, a.rope, tid, 128);
        stage_tile(sdO, a.dout + ((long)b * a.T + q0) * a.lddo + h * HD, a.lddo, nq, q0, nullptr, tid, 128);
        __syncthreads();
        // S = Q K^T and dP = dO V^T for this warp's 16 query rows
        float s[8][4], dp[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) s[i][e] = dp[i][e] = 0.f;
#pragma unroll
        for (int kc = 0; kc < 4; ++kc) {
            uint32_t qa[4], da[4];
            ldsm_x4(qa[0], qa[1], qa[2], qa[3], sQ + (warp * 16 + lr + 8 * (lsel & 1)) * LDS + kc * 16 + 8 * (lsel >> 1));
            ldsm_x4(da[0], da[1], da[2], da[3], sdO + (warp * 16 + lr + 8 * (lsel & 1)) * LDS + kc * 16 + 8 * (lsel >> 1));
#pragma unroll
            for (int nj = 0; nj < 4; ++nj) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(b0, b1, b2, b3, sK + (nj * 16 + lr + 8 * (lsel >> 1)) * LDS + kc * 16 + 8 * (lsel & 1));
                mma_bf16(s[2 * nj], qa, b0, b1);
                mma_bf16(s[2 * nj + 1], qa, b2, b3);
                ldsm_x4(b0, b1, b2, b3, sV + (nj * 16 + lr + 8 * (lsel >> 1)) * LDS + kc * 16 + 8 * (lsel & 1));
                mma_bf16(dp[2 * nj], da, b0, b1);
                mma_bf16(dp[2 * nj + 1], da, b2, b3);
            }
        }
        float lse[2], dd[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int i = q0 + warp * 16 + g + 8 * hh;
            const bool rv = i < a.T;
            lse[hh] = rv ? a.lse[((long)b * a.H + h) * a.T + i] : 0.f;
            dd[hh] = rv ? a.dvec[((long)b * a.H + h) * a.T + i] : 0.f;
        }
#pragma unroll
        for (int ni = 0; ni < 8; ++ni)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = k0 + ni * 8 + 2 * q + (e & 1);
                const int i = q0 + warp * 16 + g + 8 * (e >> 1);
                const bool ok = i < a.T && j < kv_end && (!a.causal || j <= i);
                const float p = ok ? exp2f(s[ni][e] * sl2 - lse[e >> 1]) : 0.f;
                s[ni][e] = p;
                dp[ni][e] = p * (dp[ni][e] - dd[e >> 1]);
            }
        // P and dS to smem (rows of this warp), as bf16
#pragma unroll
        for (int ni = 0; ni < 8; ++ni)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int r = warp * 16 + g + 8 * hh, c = ni * 8 + 2 * q;
                *reinterpret_cast<uint32_t*>(sP + r * LDS + c) = pack_bf16(s[ni][2 * hh], s[ni][2 * hh + 1]);
                *reinterpret_cast<uint32_t*>(sdS + r * LDS + c) = pack_bf16(dp[ni][2 * hh], dp[ni][2 * hh + 1]);
            }
        // dQ(16 rows) = dS(16 x 64 keys) K(64 keys x 64 d)
        {
            float dq[8][4];
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int e = 0; e < 4; ++e) dq[i][e] = 0.f;
#pragma unroll
            for (int kc = 0; kc < 4; ++kc) {
                uint32_t pa[4];
                pa[0] = pack_bf16(dp[2 * kc][0], dp[2 * kc][1]);
                pa[1] = pack_bf16(dp[2 * kc][2], dp[2 * kc][3]);
                pa[2] = pack_bf16(dp[2 * kc + 1][0], dp[2 * kc + 1][1]);
                pa[3] = pack_bf16(dp[2 * kc + 1][2], dp[2 * kc + 1][3]);
#pragma unroll
                for (int nj = 0; nj < 4; ++nj) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(b0, b1, b2, b3, sK + (kc * 16 + lr + 8 * (lsel & 1)) * LDS + nj * 16 + 8 * (lsel >> 1));
                    mma_bf16(dq[2 * nj], pa, b0, b1);
                    mma_bf16(dq[2 * nj + 1], pa, b2, b3);
                }
            }
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int i = q0 + warp * 16 + g + 8 * hh;
                if (i >= a.T) continue;
                float* dst = a.dq_acc + ((long)b * a.T + i) * a.ldq_acc + h * HD;
#pragma unroll
                for (int ni = 0; ni < 8; ++ni) {
                    atomicAdd(dst + ni * 8 + 2 * q, dq[ni][2 * hh] * a.scale);
                    atomicAdd(dst + ni * 8 + 2 * q + 1, dq[ni][2 * hh + 1] * a.scale);
                }
            }
        }
        __syncthreads();
        // dV(16 keys of this warp) += P^T dO ; dK += dS^T Q
#pragma unroll
        for (int kc = 0; kc < 4; ++kc) {  // over query chunks of 16
            uint32_t pa[4], sa[4];
            ldsm_x4_t(pa[0], pa[1], pa[2], pa[3], sP + (kc * 16 + lr + 8 * (lsel >> 1)) * LDS + warp * 16 + 8 * (lsel & 1));
            ldsm_x4_t(sa[0], sa[1], sa[2], sa[3], sdS + (kc * 16 + lr + 8 * (lsel >> 1)) * LDS + warp * 16 + 8 * (lsel & 1));
#pragma unroll
            for (int nj = 0; nj < 4; ++nj) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(b0, b1, b2, b3, sdO + (kc * 16 + lr + 8 * (lsel & 1)) * LDS + nj * 16 + 8 * (lsel >> 1));
                mma_bf16(dv[2 * nj], pa, b0, b1);
                mma_bf16(dv[2 * nj + 1], pa, b2, b3);
                ldsm_x4_t(b0, b1, b2, b3, sQ + (kc * 16 + lr + 8 * (lsel & 1)) * LDS + nj * 16 + 8 * (lsel >> 1));
                mma_bf16(dk[2 * nj], sa, b0, b1);
                mma_bf16(dk[2 * nj + 1], sa, b2, b3);
            }
        }
    }
    // epilogue: dK (unrotate), dV, DoRA column factors
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int jl = warp * 16 + g + 8 * hh;
        const int j = k0 + jl;
        if (j >= a.Tk) continue;
        bf16* dkr = a.dk + ((long)b * a.Tk + j) * a.lddk + h * HD;
        bf16* dvr = a.dv + ((long)b * a.Tk + j) * a.lddv + h * HD;
#pragma unroll
        for (int ni = 0; ni < 8; ++ni) {
            const int c = ni * 8 + 2 * q;
            float x0 = dk[ni][2 * hh] * a.scale, x1 = dk[ni][2 * hh + 1] * a.scale;
            if (a.rope) {
                const float2 t = reinterpret_cast<const float2*>(a.rope)[(long)j * 32 + c / 2];
                const float y0 = x0 * t.x + x1 * t.y, y1 = -x0 * t.y + x1 * t.x;
                x0 = y0;
                x1 = y1;
            }
            float v0 = dv[ni][2 * hh], v1 = dv[ni][2 * hh + 1];
            if (a.kscale) {
                x0 *= a.kscale[h * HD + c];
                x1 *= a.kscale[h * HD + c + 1];
            }
            if (a.vscale) {
                v0 *= a.vscale[h * HD + c];
                v1 *= a.vscale[h * HD + c + 1];
            }
            *reinterpret_cast<uint32_t*>(dkr + c) = pack_bf16(x0, x1);
            *reinterpret_cast<uint32_t*>(dvr + c) = pack_bf16(v0, v1);
        }
    }
}

__global__ void attn_dq_finish_kernel(const AttnArgs a, bf16* dq, long lddq, const float* qscale) {
    const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;  // one pair per thread
    const long rows = (long)a.clips * a.T;
    const int pairs = a.H * HD / 2;
    if (idx >= rows * pairs) return;
    const long row = idx / pairs;
    const int pc = (int)(idx % pairs), c = pc * 2;
    const float* src = a.dq_acc + row * a.ldq_acc + c;
    float x0 = src[0], x1 = src[1];
    if (a.rope) {
        const int pos = (int)(row % a.T);
        const float2 t = reinterpret_cast<const float2*>(a.rope)[(long)pos * 32 + (c % HD) / 2];
        const float y0 = x0 * t.x + x1 * t.y, y1 = -x0 * t.y + x1 * t.x;
        x0 = y0;
        x1 = y1;
    }
    if (qscale) {
        x0 *= qscale[c];
        x1 *= qscale[c + 1];
    }
    *reinterpret_cast<uint32_t*>(dq + row * lddq + c) = pack_bf16(x0, x1);
}

}  // namespace

void attn_fwd(const AttnArgs& a, cudaStream_t s) {
    dim3 grid((a.T + BQ - 1) / BQ, a.H, a.clips);
    attn_fwd_kernel<<<grid, 128, 0, s>>>(a);
}

void attn_bwd(const AttnArgs& a, cudaStream_t s) {
    const long warps = (long)a.clips * a.T * a.H;
    attn_dvec_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(a);
    const int smem = (2 * BKV + 4 * BQ) * LDS * 2;
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        configured = true;
    }
    dim3 grid((a.Tk + BKV - 1) / BKV, a.H, a.clips);
    attn_bwd_kernel<<<grid, 128, smem, s>>>(a);
}

void attn_dq_finish(const AttnArgs& a, bf16* dq, long lddq, const float* qscale, cudaStream_t s) {
    const long n = (long)a.clips * a.T * a.H * HD / 2;
    attn_dq_finish_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(a, dq, lddq, qscale);
}

}  // namespace act
