// attention.cu -- flash-style attention forward/backward for head_dim 64.
//
// Restates the training attention of src/ac/transformer.h:108-125 (dense softmax(scale K^T Q
// + mask) V with an optional prepended zero key, src/ac/transformer.h:74-79) without ever
// materialising the probabilities:
//   * the zero key is implicit: it starts the running max at 0 and the running sum at 1
//     (score 0, value 0), so it only enters through the log-sum-exp;
//   * masks are per-clip valid-key counts (the reference's -inf columns beyond
//     valid_tokens, src/mf/train.h:169-175) and an optional causal mask (src/mg/train.h:209-213);
//   * RoPE with stored frequencies (src/ac/transformer.h:55-61): the training step rotates q
//     and k in the projection epilogue, so these kernels read rotated inputs and only undo the
//     rotation on dQ / dK; with rope_load set (stand-alone entry points) they rotate while
//     staging tiles instead.
// Forward: 128 queries per CTA (8 warps x 16 rows), K/V tiles of 64 keys double-buffered with
// cp.async, online softmax in base 2.  Backward (recompute): one CTA per 64-key block, warps
// own 16 keys each, so P^T and dS^T stay in registers for dV += P^T dO and dK += dS^T Q; dS^T
// goes through shared memory once for dQ = dS K, accumulated with fp32 atomics.  Q / dO / LSE / D
// tiles of the next query block are prefetched while the current one is processed.
#include "common.cuh"
#include "kernels.h"

#include <stdexcept>

namespace act {

namespace {

constexpr int HD = 64;
constexpr int BKV = 64;
constexpr int LDS = HD + 8;
constexpr float LOG2E = 1.4426950408889634f;

// Synchronous staging of a [64 rows][64] f16 tile, rotating pairs when rope != nullptr.
__device__ __forceinline__ void stage_tile_sync(f16* sm, const f16* g, long ld, int nrows, int pos0,
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
                    const float2 xx = unpack_f16(w[j]);
                    const float x0 = xx.x, x1 = xx.y;
                    const float2 t = cs[j];
                    w[j] = pack_f16(x0 * t.x - x1 * t.y, x0 * t.y + x1 * t.x);
                }
            }
        }
        *reinterpret_cast<uint4*>(sm + r * LDS + ch * 8) = v;
    }
}

// Asynchronous staging of a [64 rows][64] f16 tile (rows >= nrows zero-filled).
__device__ __forceinline__ void stage_tile_async(f16* sm, const f16* g, long ld, int nrows, int tid, int nthreads) {
    for (int c = tid; c < 64 * 8; c += nthreads) {
        const int r = c >> 3, ch = c & 7;
        const bool ok = r < nrows;
        cp_async16(sm + r * LDS + ch * 8, ok ? g + (long)r * ld + ch * 8 : g, ok);
    }
}

template <bool ROPE_LOAD>
__device__ __forceinline__ void stage_tile(f16* sm, const f16* g, long ld, int nrows, int pos0, const float* rope,
                                           int tid, int nthreads) {
    if (ROPE_LOAD) stage_tile_sync(sm, g, ld, nrows, pos0, rope, tid, nthreads);
    else stage_tile_async(sm, g, ld, nrows, tid, nthreads);
}

// ---------------------------------------------------------------------------------------
// forward

constexpr int FWD_WARPS = 8;
constexpr int FWD_BQ = FWD_WARPS * 16;
constexpr int FWD_SMEM = (FWD_BQ + 4 * BKV) * LDS * 2;

template <bool ROPE_LOAD>
__global__ void __launch_bounds__(FWD_WARPS * 32) attn_fwd_kernel(const AttnArgs a) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(16) unsigned char smraw[];
    f16* sQ = reinterpret_cast<f16*>(smraw);
    f16* sK = sQ + FWD_BQ * LDS;  // [2][64][LDS]
    f16* sV = sK + 2 * BKV * LDS;  // [2][64][LDS]
    constexpr int NT = FWD_WARPS * 32;
    const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, q = lane & 3, lr = lane & 7, lsel = lane >> 3;
    const int q0 = qb * FWD_BQ;
    const int nq = min(FWD_BQ, a.T - q0);
    int kv_end = a.Tk;
    if (a.nvalid) kv_end = min(kv_end, a.nvalid[b]);
    if (a.causal) kv_end = min(kv_end, q0 + FWD_BQ);
    const float* rope_load = ROPE_LOAD ? a.rope : nullptr;

    const f16* qg = a.q + ((long)b * a.T + q0) * a.ldq + h * HD;
    stage_tile<ROPE_LOAD>(sQ, qg, a.ldq, nq, q0, rope_load, tid, NT);
    stage_tile<ROPE_LOAD>(sQ + 64 * LDS, qg + 64 * a.ldq, a.ldq, nq - 64, q0 + 64, rope_load, tid, NT);
    const int nkb = (kv_end + BKV - 1) / BKV;
    auto load_kv = [&](int kb, int buf) {
        const int k0 = kb * BKV;
        const int nk = min(BKV, kv_end - k0);
        stage_tile<ROPE_LOAD>(sK + buf * BKV * LDS, a.k + ((long)b * a.Tk + k0) * a.ldk + h * HD, a.ldk, nk, k0,
                              rope_load, tid, NT);
        stage_tile_async(sV + buf * BKV * LDS, a.v + ((long)b * a.Tk + k0) * a.ldv + h * HD, a.ldv, nk, tid, NT);
    };
    if (nkb > 0) load_kv(0, 0);
    cp_async_commit();

    const float sl2 = a.scale * LOG2E;
    float mrow[2], lrow[2];
    mrow[0] = mrow[1] = a.zero_key ? 0.f : -INFINITY;
    lrow[0] = lrow[1] = a.zero_key ? 1.f : 0.f;
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[i][e] = 0.f;
    uint32_t qf[4][4];

    for (int kb = 0; kb < nkb; ++kb) {
        const int buf = kb & 1;
        if (kb + 1 < nkb) load_kv(kb + 1, buf ^ 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        if (kb == 0) {
#pragma unroll
            for (int kc = 0; kc < 4; ++kc)
                ldsm_x4(qf[kc][0], qf[kc][1], qf[kc][2], qf[kc][3],
                        sQ + (warp * 16 + lr + 8 * (lsel & 1)) * LDS + kc * 16 + 8 * (lsel >> 1));
        }
        const f16* cK = sK + buf * BKV * LDS;
        const f16* cV = sV + buf * BKV * LDS;
        const int k0 = kb * BKV;
        const int nvk = kv_end - k0;  // keys of this block in range (>= 1): groups of 16 past them are skipped
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) s[i][e] = 0.f;
#pragma unroll
        for (int kc = 0; kc < 4; ++kc)
#pragma unroll
            for (int nj = 0; nj < 4; ++nj) {
                if (nj * 16 >= nvk) continue;  // masked below
                uint32_t b0, b1, b2, b3;
                ldsm_x4(b0, b1, b2, b3, cK + (nj * 16 + lr + 8 * (lsel >> 1)) * LDS + kc * 16 + 8 * (lsel & 1));
                mma_sync_f16(s[2 * nj], qf[kc], b0, b1);
                mma_sync_f16(s[2 * nj + 1], qf[kc], b2, b3);
            }
        float mx[2] = {-INFINITY, -INFINITY};
        const bool full = (k0 + BKV <= kv_end) && (!a.causal || k0 + BKV - 1 <= q0 + warp * 16);
#pragma unroll
        for (int ni = 0; ni < 8; ++ni)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                bool ok = true;
                if (!full) {
                    const int j = k0 + ni * 8 + 2 * q + (e & 1);
                    const int i = q0 + warp * 16 + g + 8 * (e >> 1);
                    ok = j < kv_end && (!a.causal || j <= i);
                }
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
            if (kc * 16 >= nvk) continue;  // these probabilities are zero
            uint32_t pa[4];
            pa[0] = pack_f16(s[2 * kc][0], s[2 * kc][1]);
            pa[1] = pack_f16(s[2 * kc][2], s[2 * kc][3]);
            pa[2] = pack_f16(s[2 * kc + 1][0], s[2 * kc + 1][1]);
            pa[3] = pack_f16(s[2 * kc + 1][2], s[2 * kc + 1][3]);
#pragma unroll
            for (int nj = 0; nj < 4; ++nj) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(b0, b1, b2, b3, cV + (kc * 16 + lr + 8 * (lsel & 1)) * LDS + nj * 16 + 8 * (lsel >> 1));
                mma_sync_f16(o[2 * nj], pa, b0, b1);
                mma_sync_f16(o[2 * nj + 1], pa, b2, b3);
            }
        }
        __syncthreads();  // this buffer is refilled by the prefetch of iteration kb + 2
    }
    if (nkb == 0) {  // no key in range: only the zero key (if any) contributes
        cp_async_wait<0>();
        __syncthreads();
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int i = q0 + warp * 16 + g + 8 * hh;
        if (i >= a.T) continue;
        const float inv = lrow[hh] > 0.f ? 1.f / lrow[hh] : 0.f;
        f16* orow = a.o + ((long)b * a.T + i) * a.ldo + h * HD;
#pragma unroll
        for (int ni = 0; ni < 8; ++ni)
            *reinterpret_cast<uint32_t*>(orow + ni * 8 + 2 * q) =
                pack_f16(o[ni][2 * hh] * inv, o[ni][2 * hh + 1] * inv);
        if (q == 0) {
            const float mfin = mrow[hh] == -INFINITY ? 0.f : mrow[hh];
            a.lse[((long)b * a.H + h) * a.T + i] = mfin + log2f(lrow[hh]);
        }
    }
}

// ---------------------------------------------------------------------------------------
// D[b][h][i] = sum_d dO * O : 8 threads per (row, head), one 16-byte load each.
__global__ void attn_dvec_kernel(const AttnArgs a) {
    pdl_wait();
    pdl_trigger();
    const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const long rows = (long)a.clips * a.T;
    const long per_row = (long)a.H * 8;
    const bool valid = t < rows * per_row;
    const long row = valid ? t / per_row : 0;
    const int rem = (int)(t % per_row), h = rem >> 3, part = rem & 7;
    float v = 0.f;
    if (valid) {
        const uint4 oo = *reinterpret_cast<const uint4*>(a.o + row * a.ldo + h * HD + part * 8);
        const uint4 dd = *reinterpret_cast<const uint4*>(a.dout + row * a.lddo + h * HD + part * 8);
        const uint32_t ow[4] = {oo.x, oo.y, oo.z, oo.w}, dw[4] = {dd.x, dd.y, dd.z, dd.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 o2 = unpack_f16(ow[j]), d2 = unpack_f16(dw[j]);
            v += o2.x * d2.x + o2.y * d2.y;
        }
    }
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    if (valid && part == 0) {
        const int b = (int)(row / a.T), i = (int)(row % a.T);
        a.dvec[((long)b * a.H + h) * a.T + i] = v;
    }
}

// ---------------------------------------------------------------------------------------
// backward

constexpr int BWD_BQ = 64;
constexpr int BWD_SMEM = (2 * BKV + 4 * BWD_BQ + BKV) * LDS * 2 + 4 * BWD_BQ * 4;

template <bool ROPE_LOAD>
__global__ void __launch_bounds__(128) attn_bwd_kernel(const AttnArgs a) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(16) unsigned char smraw[];
    f16* sK = reinterpret_cast<f16*>(smraw);
    f16* sV = sK + BKV * LDS;
    f16* sQ = sV + BKV * LDS;          // [2][64][LDS]
    f16* sdO = sQ + 2 * BWD_BQ * LDS;  // [2][64][LDS]
    f16* sdS = sdO + 2 * BWD_BQ * LDS; // [64 keys][LDS]  dS^T
    float* sL = reinterpret_cast<float*>(sdS + BKV * LDS);  // [2][64] lse
    float* sD = sL + 2 * BWD_BQ;                             // [2][64] rowsum(dO*O)
    const int kb = blockIdx.x / a.qsplit, part = blockIdx.x % a.qsplit, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, q = lane & 3, lr = lane & 7, lsel = lane >> 3;
    const int k0 = kb * BKV;
    int kv_end = a.Tk;
    if (a.nvalid) kv_end = min(kv_end, a.nvalid[b]);
    const int nk = max(0, min(BKV, kv_end - k0));
    const float* rope_load = ROPE_LOAD ? a.rope : nullptr;

    stage_tile<ROPE_LOAD>(sK, a.k + ((long)b * a.Tk + k0) * a.ldk + h * HD, a.ldk, nk, k0, rope_load, tid, 128);
    stage_tile_async(sV, a.v + ((long)b * a.Tk + k0) * a.ldv + h * HD, a.ldv, nk, tid, 128);

    const int qb0 = a.causal ? k0 / BWD_BQ : 0;
    const int nqb = (a.T + BWD_BQ - 1) / BWD_BQ;
    // without keys in range the CTA has nothing to add, except when it writes dQ directly: then
    // its query blocks still run (every score masked, dQ exactly zero) so that their rows are written
    const int qb_all = (nk > 0 || a.dq_h) ? qb0 : nqb;
    // this CTA's share of the key block's query blocks
    const int qb_first = qb_all + (int)((long)(nqb - qb_all) * part / a.qsplit);
    const int qb_end = qb_all + (int)((long)(nqb - qb_all) * (part + 1) / a.qsplit);
    auto load_q = [&](int qb, int buf) {
        const int q0 = qb * BWD_BQ;
        const int nq = min(BWD_BQ, a.T - q0);
        stage_tile<ROPE_LOAD>(sQ + buf * BWD_BQ * LDS, a.q + ((long)b * a.T + q0) * a.ldq + h * HD, a.ldq, nq, q0,
                              rope_load, tid, 128);
        stage_tile_async(sdO + buf * BWD_BQ * LDS, a.dout + ((long)b * a.T + q0) * a.lddo + h * HD, a.lddo, nq, tid, 128);
        if (tid < 32) {  // 16 x 16 bytes of lse, 16 x 16 bytes of D
            const int c = tid & 15;
            const bool ok = c * 4 < nq;
            const float* src = (tid < 16 ? a.lse : a.dvec) + ((long)b * a.H + h) * a.T + q0 + c * 4;
            float* dst = (tid < 16 ? sL : sD) + buf * BWD_BQ + c * 4;
            const bool full = ok && (q0 + c * 4 + 4 <= a.T) && ((reinterpret_cast<uintptr_t>(src) & 15) == 0);
            if (full) cp_async16(dst, src, true);
            else
                for (int j = 0; j < 4; ++j) dst[j] = (q0 + c * 4 + j < a.T) ? src[j] : 0.f;
        }
    };
    if (qb_first < qb_end) load_q(qb_first, 0);
    cp_async_commit();
    // a warp owns keys k0 + 16 warp .. +15; with none of them in range (few keys, e.g. the 32
    // conditioning tokens in a 64-key block) its scores, dV / dK and dS^T rows are all zero: it
    // skips that work and its dS^T rows are cleared once for the dQ product
    const bool live = warp * 16 < nk;
    if (!live)
        for (int c = lane; c < 16 * (HD / 8); c += 32)
            *reinterpret_cast<uint4*>(sdS + (warp * 16 + c / (HD / 8)) * LDS + (c % (HD / 8)) * 8) = make_uint4(0, 0, 0, 0);

    const float sl2 = a.scale * LOG2E;
    float dk[8][4], dv[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

    for (int qb = qb_first, it = 0; qb < qb_end; ++qb, ++it) {
        const int buf = it & 1;
        if (qb + 1 < qb_end) load_q(qb + 1, buf ^ 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const int q0 = qb * BWD_BQ;
        const f16* cQ = sQ + buf * BWD_BQ * LDS;
        const f16* cdO = sdO + buf * BWD_BQ * LDS;
        const float* cL = sL + buf * BWD_BQ;
        const float* cD = sD + buf * BWD_BQ;
        // S^T = K Q^T and dP^T = V dO^T for this warp's 16 keys x 64 queries
        float s[8][4], dp[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) s[i][e] = dp[i][e] = 0.f;
        if (live) {
#pragma unroll
        for (int kc = 0; kc < 4; ++kc) {
            uint32_t ka[4], va[4];
            ldsm_x4(ka[0], ka[1], ka[2], ka[3], sK + (warp * 16 + lr + 8 * (lsel & 1)) * LDS + kc * 16 + 8 * (lsel >> 1));
            ldsm_x4(va[0], va[1], va[2], va[3], sV + (warp * 16 + lr + 8 * (lsel & 1)) * LDS + kc * 16 + 8 * (lsel >> 1));
#pragma unroll
            for (int nj = 0; nj < 4; ++nj) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(b0, b1, b2, b3, cQ + (nj * 16 + lr + 8 * (lsel >> 1)) * LDS + kc * 16 + 8 * (lsel & 1));
                mma_sync_f16(s[2 * nj], ka, b0, b1);
                mma_sync_f16(s[2 * nj + 1], ka, b2, b3);
                ldsm_x4(b0, b1, b2, b3, cdO + (nj * 16 + lr + 8 * (lsel >> 1)) * LDS + kc * 16 + 8 * (lsel & 1));
                mma_sync_f16(dp[2 * nj], va, b0, b1);
                mma_sync_f16(dp[2 * nj + 1], va, b2, b3);
            }
        }
        const bool full = (q0 + BWD_BQ <= a.T) && (k0 + BKV <= kv_end) && (!a.causal || k0 + BKV - 1 <= q0);
#pragma unroll
        for (int ni = 0; ni < 8; ++ni)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int il = ni * 8 + 2 * q + (e & 1);  // query within the block (column)
                bool ok = true;
                if (!full) {
                    const int i = q0 + il;
                    const int j = k0 + warp * 16 + g + 8 * (e >> 1);
                    ok = i < a.T && j < kv_end && (!a.causal || j <= i);
                }
                const float p = ok ? exp2f(s[ni][e] * sl2 - cL[il]) : 0.f;
                s[ni][e] = p;
                dp[ni][e] = p * (dp[ni][e] - cD[il]);
            }
        }  // live
        // dV += P^T dO ; dK += dS^T Q  (A operands straight from the accumulators)
#pragma unroll
        for (int kc = 0; kc < 4; ++kc) {
            if (!live) break;
            uint32_t pa[4], sa[4];
            pa[0] = pack_f16(s[2 * kc][0], s[2 * kc][1]);
            pa[1] = pack_f16(s[2 * kc][2], s[2 * kc][3]);
            pa[2] = pack_f16(s[2 * kc + 1][0], s[2 * kc + 1][1]);
            pa[3] = pack_f16(s[2 * kc + 1][2], s[2 * kc + 1][3]);
            sa[0] = pack_f16(dp[2 * kc][0], dp[2 * kc][1]);
            sa[1] = pack_f16(dp[2 * kc][2], dp[2 * kc][3]);
            sa[2] = pack_f16(dp[2 * kc + 1][0], dp[2 * kc + 1][1]);
            sa[3] = pack_f16(dp[2 * kc + 1][2], dp[2 * kc + 1][3]);
#pragma unroll
            for (int nj = 0; nj < 4; ++nj) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(b0, b1, b2, b3, cdO + (kc * 16 + lr + 8 * (lsel & 1)) * LDS + nj * 16 + 8 * (lsel >> 1));
                mma_sync_f16(dv[2 * nj], pa, b0, b1);
                mma_sync_f16(dv[2 * nj + 1], pa, b2, b3);
                ldsm_x4_t(b0, b1, b2, b3, cQ + (kc * 16 + lr + 8 * (lsel & 1)) * LDS + nj * 16 + 8 * (lsel >> 1));
                mma_sync_f16(dk[2 * nj], sa, b0, b1);
                mma_sync_f16(dk[2 * nj + 1], sa, b2, b3);
            }
            // dS^T rows of this warp to shared memory for dQ
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int r = warp * 16 + g + 8 * hh;
                *reinterpret_cast<uint32_t*>(sdS + r * LDS + kc * 16 + 2 * q) = sa[hh];
                *reinterpret_cast<uint32_t*>(sdS + r * LDS + kc * 16 + 8 + 2 * q) = sa[2 + hh];
            }
        }
        __syncthreads();
        // dQ (16 queries of this warp x 64 d) = dS K, summed over this CTA's 64 keys
        {
            float dq[8][4];
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int e = 0; e < 4; ++e) dq[i][e] = 0.f;
#pragma unroll
            for (int kc = 0; kc < 4; ++kc) {
                uint32_t da[4];
                ldsm_x4_t(da[0], da[1], da[2], da[3], sdS + (kc * 16 + lr + 8 * (lsel >> 1)) * LDS + warp * 16 + 8 * (lsel & 1));
#pragma unroll
                for (int nj = 0; nj < 4; ++nj) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(b0, b1, b2, b3, sK + (kc * 16 + lr + 8 * (lsel & 1)) * LDS + nj * 16 + 8 * (lsel >> 1));
                    mma_sync_f16(dq[2 * nj], da, b0, b1);
                    mma_sync_f16(dq[2 * nj + 1], da, b2, b3);
                }
            }
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int i = q0 + warp * 16 + g + 8 * hh;
                if (i >= a.T) continue;
                float* dst = a.dq_acc + ((long)b * a.T + i) * a.ldq_acc + h * HD;
                // with a single key block this CTA is the only contributor to these rows
                if (a.dq_h) {
                    f16* db = a.dq_h + ((long)b * a.T + i) * a.lddq_h + h * HD;
#pragma unroll
                    for (int ni = 0; ni < 8; ++ni) {
                        const int c = ni * 8 + 2 * q;
                        float x0 = dq[ni][2 * hh] * a.scale, x1 = dq[ni][2 * hh + 1] * a.scale;
                        if (a.dq_scale) {
                            x0 *= a.dq_scale[h * HD + c];
                            x1 *= a.dq_scale[h * HD + c + 1];
                        }
                        *reinterpret_cast<uint32_t*>(db + c) = pack_f16(x0, x1);
                    }
                } else if (a.Tk <= BKV) {
#pragma unroll
                    for (int ni = 0; ni < 8; ++ni)
                        *reinterpret_cast<float2*>(dst + ni * 8 + 2 * q) =
                            make_float2(dq[ni][2 * hh] * a.scale, dq[ni][2 * hh + 1] * a.scale);
                } else {
#pragma unroll
                    for (int ni = 0; ni < 8; ++ni)
                        atomicAdd(reinterpret_cast<float2*>(dst + ni * 8 + 2 * q),
                                  make_float2(dq[ni][2 * hh] * a.scale, dq[ni][2 * hh + 1] * a.scale));
                }
            }
        }
        __syncthreads();  // sdS and this Q/dO buffer are rewritten next
    }
    cp_async_wait<0>();
    if (!a.dk && !a.dk_acc) return;  // dQ only (nothing consumes dK / dV)
    // epilogue: dK (unrotate), dV, DoRA column factors
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int jl = warp * 16 + g + 8 * hh;
        const int j = k0 + jl;
        if (j >= a.Tk) continue;
        f16* dkr = a.dk + ((long)b * a.Tk + j) * a.lddk + h * HD;
        f16* dvr = a.dv + ((long)b * a.Tk + j) * a.lddv + h * HD;
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
            if (a.dk_acc) {  // partial over this CTA's query blocks, in its own slice (zero if it had none)
                const long r = ((long)part * a.clips * a.Tk + (long)b * a.Tk + j) * a.H * HD + h * HD + c;
                *reinterpret_cast<float2*>(a.dk_acc + r) = make_float2(x0, x1);
                *reinterpret_cast<float2*>(a.dv_acc + r) = make_float2(v0, v1);
            } else {
                *reinterpret_cast<uint32_t*>(dkr + c) = pack_f16(x0, x1);
                *reinterpret_cast<uint32_t*>(dvr + c) = pack_f16(v0, v1);
            }
        }
    }
}

// dk / dv (f16) from the fp32 partials of a query-split backward, added in split order (the
// same sum whichever CTA finished first): 4 floats per thread
__global__ void attn_dkv_finish_kernel(const AttnArgs a) {
    pdl_wait();
    pdl_trigger();
    const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const int quads = a.H * HD / 4;
    const long rows = (long)a.clips * a.Tk;
    if (idx >= rows * quads) return;
    const long row = idx / quads;
    const int c = (int)(idx % quads) * 4;
    float4 k = make_float4(0.f, 0.f, 0.f, 0.f), v = k;
    for (int q = 0; q < a.qsplit; ++q) {
        const long at = ((long)q * rows + row) * a.H * HD + c;
        const float4 kq = *reinterpret_cast<const float4*>(a.dk_acc + at);
        const float4 vq = *reinterpret_cast<const float4*>(a.dv_acc + at);
        k.x += kq.x; k.y += kq.y; k.z += kq.z; k.w += kq.w;
        v.x += vq.x; v.y += vq.y; v.z += vq.z; v.w += vq.w;
    }
    *reinterpret_cast<uint2*>(a.dk + row * a.lddk + c) = make_uint2(pack_f16(k.x, k.y), pack_f16(k.z, k.w));
    *reinterpret_cast<uint2*>(a.dv + row * a.lddv + c) = make_uint2(pack_f16(v.x, v.y), pack_f16(v.z, v.w));
}

// dq (f16) = unrotate(dq_acc) * qscale : 4 floats per thread
__global__ void attn_dq_finish_kernel(const AttnArgs a, f16* dq, long lddq, const float* qscale) {
    pdl_wait();
    pdl_trigger();
    const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const long rows = (long)a.clips * a.T;
    const int quads = a.H * HD / 4;
    if (idx >= rows * quads) return;
    const long row = idx / quads;
    const int c = (int)(idx % quads) * 4;
    const float4 v = *reinterpret_cast<const float4*>(a.dq_acc + row * a.ldq_acc + c);
    float x[4] = {v.x, v.y, v.z, v.w};
    if (a.rope) {
        const int pos = (int)(row % a.T);
        const float2* t = reinterpret_cast<const float2*>(a.rope) + (long)pos * 32 + (c % HD) / 2;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float x0 = x[2 * j], x1 = x[2 * j + 1];
            x[2 * j] = x0 * t[j].x + x1 * t[j].y;
            x[2 * j + 1] = -x0 * t[j].y + x1 * t[j].x;
        }
    }
    if (qscale)
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] *= qscale[c + j];
    *reinterpret_cast<uint2*>(dq + row * lddq + c) = make_uint2(pack_f16(x[0], x[1]), pack_f16(x[2], x[3]));
}

template <class K>
void set_smem(K kern, int bytes) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

}  // namespace

void attn_fwd(const AttnArgs& a, cudaStream_t s) {
    static DeviceOnce once;
    once([] {
        set_smem(attn_fwd_kernel<true>, FWD_SMEM);
        set_smem(attn_fwd_kernel<false>, FWD_SMEM);
    });
    dim3 grid((a.T + FWD_BQ - 1) / FWD_BQ, a.H, a.clips);
    if (a.rope && a.rope_load) launch_pdl(attn_fwd_kernel<true>, grid, dim3(FWD_WARPS * 32), FWD_SMEM, s, a);
    else launch_pdl(attn_fwd_kernel<false>, grid, dim3(FWD_WARPS * 32), FWD_SMEM, s, a);
}

void attn_dvec(const AttnArgs& a, cudaStream_t s) {
    const long threads = (long)a.clips * a.T * a.H * 8;
    launch_pdl(attn_dvec_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, s, a);
}

void attn_bwd(const AttnArgs& a, cudaStream_t s) {
    attn_dvec(a, s);
    static DeviceOnce once;
    once([] {
        set_smem(attn_bwd_kernel<true>, BWD_SMEM);
        set_smem(attn_bwd_kernel<false>, BWD_SMEM);
    });
    if (a.qsplit < 1 || (a.qsplit > 1 && a.dk && (!a.dk_acc || !a.dv_acc)))
        throw std::runtime_error("attn_bwd: query split with dK / dV needs dk_acc / dv_acc");
    if (a.dq_h && (a.Tk > BKV || a.rope || a.lddq_h % 2 || (reinterpret_cast<uintptr_t>(a.dq_h) & 3)))
        throw std::runtime_error("attn_bwd: direct f16 dQ needs a single key block and no RoPE");
    dim3 grid((unsigned)(((a.Tk + BKV - 1) / BKV) * a.qsplit), a.H, a.clips);
    if (a.rope && a.rope_load) launch_pdl(attn_bwd_kernel<true>, grid, dim3(128), BWD_SMEM, s, a);
    else launch_pdl(attn_bwd_kernel<false>, grid, dim3(128), BWD_SMEM, s, a);
}

void attn_dkv_finish(const AttnArgs& a, cudaStream_t s) {
    const long n = (long)a.clips * a.Tk * a.H * HD / 4;
    launch_pdl(attn_dkv_finish_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, a);
}

void attn_dq_finish(const AttnArgs& a, f16* dq, long lddq, const float* qscale, cudaStream_t s) {
    const long n = (long)a.clips * a.T * a.H * HD / 4;
    launch_pdl(attn_dq_finish_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, a, dq, lddq, qscale);
}

}  // namespace act
