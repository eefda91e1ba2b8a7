// attention_tc.cu -- self-attention forward on the tcgen05 tensor cores (head_dim 64).
//
// Same contract as attn_fwd (attention.cu): softmax(scale K^T Q + mask) V per (clip, head) with
// the optional implicit zero key (running max 0, running sum 1: src/ac/transformer.h:74-79), the
// optional causal mask (src/mg/train.h:209-213), base-2 log-sum-exp out for the backward.  Inputs
// arrive already rotated (RoPE sits in the projection epilogue).
//
// One CTA per 128 queries of one (clip, head); two CTAs per SM, so one CTA's softmax overlaps
// the other's MMAs.  Warp roles:
//   warp 0      TMA producer: Q once, then K/V blocks of 64 keys into a 4-stage ring
//               (128-byte swizzle; rows past the tensor read as zero, keys past the clip are
//               masked)
//   warp 1      MMA issuer (one thread): S = Q K^T (128 x 64, fp32, two TMEM buffers so the
//               next block's scores are computed while this block's softmax runs), then
//               O += P V (128 x 64, fp32 in TMEM) with P (f16 pairs) read from TMEM
//   warps 2..5  softmax, one query row per thread: tcgen05.ld the row of S, online softmax in
//               base 2 with a lazily updated running max (the max used for the exponentials is
//               only raised when the block maximum exceeds it by more than 2^8, which bounds
//               every probability by 256 and keeps O's rescaling off the common path), P to
//               TMEM, O rescaled in TMEM when the max moved; finally O / l and the LSE.
//
// Backward (attn_bwd_tc): one CTA per 128 keys of one (clip, head), looping over blocks of 128
// queries, with the scores recomputed in the transposed (key-major) frame:
//   S^T = K Q^T, dP^T = V dO^T            (128 x 128 each, fp32 in TMEM)
//   P^T = exp2(scale*log2e*S^T - lse), dS^T = P^T (dP^T - D)     (one key row per thread; P^T
//                                         to TMEM, dS^T to shared memory, queries contiguous)
//   dV += P^T dO, dK += dS^T Q             (fp32 accumulators stay in TMEM across the loop)
//   dQ  = dS K  (dS read back from the dS^T tile as an MN-major operand), added into the fp32
//         dQ accumulator with TMA bulk reduce-add tiles (out-of-range rows add exact zeros)
// Warp roles: 0 TMA (K, V once; Q, dO per block into 3 stages), 1 MMA issue, 2..9 P / dS in two
// groups of query columns and the final dK / dV epilogue (RoPE undone on dK, DoRA column
// factors), 10..13 the dQ epilogue.  P^T goes to TMEM as f16 pairs and is the A operand of the
// dV MMAs straight from there (released right after them); dS^T is double-buffered in shared
// memory; Q / dO have three stages, so the next-but-one block's tiles load while this one runs.
// Every mbarrier wait is bounded (globaltimer) and reports into the shared error word.
#include <cuda.h>

#include <stdexcept>
#include <string>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace act {

namespace {

using namespace tc;

constexpr int AT_BQ = 128;      // queries per CTA
constexpr int AT_BK = 64;       // keys per block
constexpr int AT_HD = 64;
constexpr int AT_QTILE = AT_BQ * AT_HD * 2;  // 16 KB: 128 rows x 64 f16 (128-byte rows)
constexpr int AT_KTILE = AT_BK * AT_HD * 2;  //  8 KB
constexpr int AT_STAGES = 4;
constexpr int AT_Q_OFF = 0;
constexpr int AT_K_OFF = AT_QTILE;                           // [AT_STAGES] stages of K
constexpr int AT_V_OFF = AT_K_OFF + AT_STAGES * AT_KTILE;    // [AT_STAGES] stages of V
constexpr int AT_BAR_OFF = AT_V_OFF + AT_STAGES * AT_KTILE;
constexpr int AT_SMEM = AT_BAR_OFF + 256 + 1024;
constexpr int AT_THREADS = 6 * 32;
constexpr uint32_t AT_TMEM_COLS = 256;       // S: columns 0..63 and 64..127, O: 128..191, P (f16 pairs): 192..223
constexpr float AT_LOG2E = 1.4426950408889634f;
constexpr float AT_RESCALE = 8.0f;           // lazy-max threshold (log2 units)

struct AtMaps {
    CUtensorMap q, k, v;
};

__device__ __forceinline__ void tmem_ld32_nw(uint32_t taddr, float* f) {
    uint32_t* r = reinterpret_cast<uint32_t*>(f);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* f) {
    const uint32_t* r = reinterpret_cast<const uint32_t*>(f);
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// D (+)= A B with A read from tensor memory (K-major: lane = row, two 16-bit K elements per
// 32-bit column) and B from shared memory
__device__ __forceinline__ void mma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ float fast_ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Packed fp32 pair arithmetic (sm_100: one instruction for two lanes' worth of FMA / ADD / MUL).
__device__ __forceinline__ unsigned long long f2_bits(float2 v) { return *reinterpret_cast<unsigned long long*>(&v); }
__device__ __forceinline__ float2 bits_f2(unsigned long long v) { return *reinterpret_cast<float2*>(&v); }
__device__ __forceinline__ float2 fma_f2(float2 a, float2 b, float2 c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
    return bits_f2(d);
}
__device__ __forceinline__ float2 add_f2(float2 a, float2 b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return bits_f2(d);
}
__device__ __forceinline__ float2 sub_f2(float2 a, float2 b) {
    unsigned long long d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return bits_f2(d);
}
__device__ __forceinline__ float2 mul_f2(float2 a, float2 b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return bits_f2(d);
}

// byte offset of 16-byte unit u of row r in a 1024-aligned, 128-byte-swizzled tile
__device__ __forceinline__ uint32_t at_sw128(int r, int u) { return r * 128 + ((u ^ (r & 7)) << 4); }

__global__ void __launch_bounds__(AT_THREADS, 2) attn_fwd_tc_kernel(const __grid_constant__ AtMaps maps,
                                                                     const AttnArgs a, int* err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023) & ~1023u;
    unsigned char* smem = smem_raw + (base - raw);
    const uint32_t bars = base + AT_BAR_OFF;
    const uint32_t q_full = bars, p_full = bars + 8, o_done = bars + 16;
    auto s_full = [&](int t) { return bars + 24 + 8 * t; };
    auto kv_full = [&](int s) { return bars + 40 + 8 * s; };
    auto kv_empty = [&](int s) { return bars + 40 + 8 * AT_STAGES + 8 * s; };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + AT_BAR_OFF + 40 + 16 * AT_STAGES);

    if (threadIdx.x == 0) {
        prefetch_tmap(&maps.q);
        prefetch_tmap(&maps.k);
        prefetch_tmap(&maps.v);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    if (a.causal) {
        // causal: query block qb visits qb + 1 key blocks.  The heaviest go first over every
        // (clip, head), so the last wave holds the lightest CTAs.
        const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z), per = gridDim.y * gridDim.z;
        qb = gridDim.x - 1 - lin / per;
        h = (lin % per) % gridDim.y;
        b = (lin % per) / gridDim.y;
    }
    const int q0 = qb * AT_BQ;
    int kv_end = a.Tk;
    if (a.nvalid) kv_end = min(kv_end, a.nvalid[b]);
    if (a.causal) kv_end = min(kv_end, q0 + AT_BQ);
    const int nkb = kv_end > 0 ? (kv_end + AT_BK - 1) / AT_BK : 0;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(s_full(0), 1);
        mbar_init(s_full(1), 1);
        mbar_init(p_full, 4);  // one arrive per softmax warp
        mbar_init(o_done, 1);
        for (int s = 0; s < AT_STAGES; ++s) {
            mbar_init(kv_full(s), 1);
            mbar_init(kv_empty(s), 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(AT_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS = tmem, tO = tmem + 2 * AT_BK, tP = tmem + 3 * AT_BK;  // S buffer t at tS + t * AT_BK
    pdl_wait();
    pdl_trigger();

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ TMA producer
        if (nkb > 0) {
            mbar_expect_tx(q_full, AT_QTILE);
            tma_load_2d(base + AT_Q_OFF, &maps.q, h * AT_HD, b * a.T + q0, q_full);
            for (int j = 0; j < nkb; ++j) {
                const int s = j % AT_STAGES;
                if (!mbar_wait(kv_empty(s), ((j / AT_STAGES) & 1) ^ 1, err, 31)) break;
                mbar_expect_tx(kv_full(s), 2 * AT_KTILE);
                tma_load_2d(base + AT_K_OFF + s * AT_KTILE, &maps.k, h * AT_HD, b * a.Tk + j * AT_BK, kv_full(s));
                tma_load_2d(base + AT_V_OFF + s * AT_KTILE, &maps.v, h * AT_HD, b * a.Tk + j * AT_BK, kv_full(s));
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ MMA issuer
        constexpr uint32_t IDESC_S = IDESC_F16_F32ACC | ((uint32_t)(AT_BK >> 3) << 17) |
                                     ((uint32_t)(AT_BQ >> 4) << 24);
        constexpr uint32_t IDESC_PV = IDESC_F16_F32ACC | (1u << 16) |
                                      ((uint32_t)(AT_HD >> 3) << 17) | ((uint32_t)(AT_BQ >> 4) << 24);
        const uint64_t dq = smem_desc(base + AT_Q_OFF, 16, 1024);
        const uint64_t dk0 = smem_desc(base + AT_K_OFF, 16, 1024);
        const uint64_t dv0 = smem_desc(base + AT_V_OFF, 8192, 1024);
        bool ok = nkb > 0 && mbar_wait(q_full, 0, err, 32);
        auto issue_s = [&](int j) {  // S[j & 1] = Q K_j^T
            const int st = j % AT_STAGES;
            if (!mbar_wait(kv_full(st), (j / AT_STAGES) & 1, err, 33)) return false;
            const uint64_t dk = dk0 + (uint64_t)((st * AT_KTILE) >> 4);
#pragma unroll
            for (int k16 = 0; k16 < AT_HD / 16; ++k16)
                mma_f16(tS + (j & 1) * AT_BK, dq + (uint64_t)(k16 * 2), dk + (uint64_t)(k16 * 2), IDESC_S,
                        k16 > 0 ? 1u : 0u);
            mma_commit(s_full(j & 1));
            return true;
        };
        if (ok) ok = issue_s(0);
        for (int j = 0; ok && j < nkb; ++j) {
            // scores of the next block while the softmax works on this one (its S buffer was
            // released by the softmax of block j - 1)
            if (j + 1 < nkb && !issue_s(j + 1)) { ok = false; break; }
            if (!mbar_wait(p_full, j & 1, err, 34)) { ok = false; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");  // P stored by the softmax
            const uint64_t dv = dv0 + (uint64_t)(((j % AT_STAGES) * AT_KTILE) >> 4);
#pragma unroll
            for (int k16 = 0; k16 < AT_BK / 16; ++k16)  // P: TMEM, 8 columns per 16 keys; V: MN-major, +16 rows
                mma_f16_ta(tO, tP + 8 * k16, dv + (uint64_t)(k16 * 128), IDESC_PV, (j > 0 || k16 > 0) ? 1u : 0u);
            mma_commit(o_done);
            mma_commit(kv_empty(j % AT_STAGES));
        }
    } else if (warp >= 2) {
        // ------------------------------------------------------------ softmax + epilogue
        const int quad = warp & 3;
        const int r = quad * 32 + lane;  // query row within the block
        const int i = q0 + r;
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        const float sl2 = a.scale * AT_LOG2E;
        float m_run = a.zero_key ? 0.f : -INFINITY;
        float l_run = a.zero_key ? 1.f : 0.f;
        bool ok = true;
        for (int j = 0; j < nkb; ++j) {
            if (lane == 0) ok = mbar_wait(s_full(j & 1), (j >> 1) & 1, err, 36);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            float s[AT_BK];
#pragma unroll
            for (int c = 0; c < AT_BK / 32; ++c) tmem_ld32_nw(tS + (j & 1) * AT_BK + lane_base + c * 32, s + c * 32);
            tmem_wait_ld();
            const int k0 = j * AT_BK;
            const bool full = k0 + AT_BK <= kv_end && (!a.causal || k0 + AT_BK - 1 <= q0);
            if (!full) {
                const int lim = min(kv_end - k0, a.causal ? i - k0 + 1 : AT_BK);  // keys c < lim are valid
#pragma unroll
                for (int c = 0; c < AT_BK; ++c)
                    if (c >= lim) s[c] = -INFINITY;
            }
            // block max of the raw scores (scale > 0), eight independent chains
            float mx[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) mx[e] = s[e];
#pragma unroll
            for (int c = 8; c < AT_BK; ++c) mx[c & 7] = fmaxf(mx[c & 7], s[c]);
            const float mb = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                   fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * sl2;
            const float m_new = fmaxf(m_run, mb);
            const bool resc = m_new > m_run + AT_RESCALE || m_run == -INFINITY;
            const float m_use = resc ? m_new : m_run;
            const float m_sub = m_use == -INFINITY ? 0.f : m_use;
            const float alpha = resc ? fast_ex2(m_run - m_sub) : 1.f;  // m_run = -inf: alpha = 0
            // exponentials and their sum on packed pairs (four independent partial sums)
            float2 sm[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) sm[e] = make_float2(0.f, 0.f);
            const float2 sl = make_float2(sl2, sl2), nm = make_float2(-m_sub, -m_sub);
#pragma unroll
            for (int c = 0; c < AT_BK; c += 2) {
                const float2 x = fma_f2(make_float2(s[c], s[c + 1]), sl, nm);
                const float2 pv = make_float2(fast_ex2(x.x), fast_ex2(x.y));
                s[c] = pv.x;
                s[c + 1] = pv.y;
                sm[(c >> 1) & 3] = add_f2(sm[(c >> 1) & 3], pv);
            }
            const float ls = ((sm[0].x + sm[0].y) + (sm[1].x + sm[1].y)) + ((sm[2].x + sm[2].y) + (sm[3].x + sm[3].y));
            l_run = l_run * alpha + ls;
            m_run = m_use;
            // PV_{j-1} has finished: O may be rescaled and the P buffer rewritten
            if (j > 0) {
                if (lane == 0) ok = mbar_wait(o_done, (j - 1) & 1, err, 37);
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                if (__any_sync(0xffffffffu, alpha != 1.f)) {
                    float o[32];
#pragma unroll
                    for (int c = 0; c < AT_HD / 32; ++c) {
                        tmem_ld32_nw(tO + lane_base + c * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] *= alpha;
                        tmem_st32(tO + lane_base + c * 32, o);
                    }
                    tmem_wait_st();
                }
            }
            {  // P of this query row as f16 pairs into TMEM, the A operand of O += P V
                uint32_t pk[AT_BK / 2];
#pragma unroll
                for (int c2 = 0; c2 < AT_BK / 2; ++c2) pk[c2] = pack_f16(s[2 * c2], s[2 * c2 + 1]);
                tmem_st32(tP + lane_base, reinterpret_cast<const float*>(pk));
                tmem_wait_st();
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        // epilogue: O / l (32 columns at a time), LSE
        bool have_o = ok && nkb > 0;
        if (have_o) {
            if (lane == 0) have_o = mbar_wait(o_done, (nkb - 1) & 1, err, 38);
            have_o = __shfl_sync(0xffffffffu, have_o ? 1 : 0, 0) != 0;
        }
        if (have_o) asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        f16* orow = a.o + ((long)b * a.T + min(i, a.T - 1)) * a.ldo + h * AT_HD;
#pragma unroll 1
        for (int c = 0; c < AT_HD / 32; ++c) {
            float o[32];
            if (have_o) {
                tmem_ld32_nw(tO + lane_base + c * 32, o);  // warp-collective: every lane takes part
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int e = 0; e < 32; ++e) o[e] = 0.f;
            }
            if (i < a.T)
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    *reinterpret_cast<uint4*>(orow + c * 32 + 8 * u) = make_uint4(
                        pack_f16(o[8 * u] * inv, o[8 * u + 1] * inv), pack_f16(o[8 * u + 2] * inv, o[8 * u + 3] * inv),
                        pack_f16(o[8 * u + 4] * inv, o[8 * u + 5] * inv), pack_f16(o[8 * u + 6] * inv, o[8 * u + 7] * inv));
        }
        if (i < a.T) {
            const float mfin = m_run == -INFINITY ? 0.f : m_run;
            a.lse[((long)b * a.H + h) * a.T + i] = mfin + __log2f(l_run);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(AT_TMEM_COLS));
}


// ---------------------------------------------------------------------------------------
// backward
constexpr int AB_BK = 128;  // keys per CTA
constexpr int AB_BQ = 128;  // queries per block
constexpr int AB_T16 = 128 * 64 * 2;         // 16 KB: a 128 x 64 f16 tile (128-byte rows)
constexpr int AB_K_OFF = 0;
constexpr int AB_V_OFF = AB_T16;
constexpr int AB_QD_STAGES = 3;
constexpr int AB_QD_OFF = 2 * AB_T16;        // [3] stages of { Q, dO }
constexpr int AB_DS_OFF = 8 * AB_T16;        // [2] buffers of dS^T: [128 keys][128 queries] as two 64-query sub-tiles
constexpr int AB_DQ_OFF = 12 * AB_T16;       // dQ staging: one [128 queries][32 fp32] sub-tile
constexpr int AB_LSE_OFF = 13 * AB_T16;      // [2] x { lse[128], D[128] } fp32
constexpr int AB_BAR_OFF = AB_LSE_OFF + 2 * 256 * 4;
constexpr int AB_SMEM = AB_BAR_OFF + 256 + 1024;
constexpr int AB_THREADS = 14 * 32;
// S^T 0..127, dP^T 128..255, dV 256..319, dK 320..383, dQ 384..447, P^T (f16 pairs) 448..511
constexpr uint32_t AB_TMEM_COLS = 512;

struct AbMaps {
    CUtensorMap q, k, v, dout, dq;
};

__global__ void __launch_bounds__(AB_THREADS, 1) attn_bwd_tc_kernel(const __grid_constant__ AbMaps maps,
                                                                     const AttnArgs a, int* err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023) & ~1023u;
    unsigned char* smem = smem_raw + (base - raw);
    const uint32_t bars = base + AB_BAR_OFF;
    // p_free: block u's dV MMAs have read P^T;  ds_free(d): the dK / dQ MMAs have read dS^T buffer d
    const uint32_t kv_full = bars, s_full = bars + 8, s_free = bars + 16, ds_full = bars + 24, p_free = bars + 32,
                   dq_full = bars + 40, dq_free = bars + 48, acc_done = bars + 56;
    auto qd_full = [&](int st) { return bars + 64 + 8 * st; };
    auto qd_empty = [&](int st) { return bars + 88 + 8 * st; };
    auto ds_free = [&](int d) { return bars + 112 + 8 * d; };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + AB_BAR_OFF + 128);

    if (threadIdx.x == 0) {
        prefetch_tmap(&maps.q);
        prefetch_tmap(&maps.k);
        prefetch_tmap(&maps.v);
        prefetch_tmap(&maps.dout);
        prefetch_tmap(&maps.dq);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int kb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    if (a.causal) {
        // causal: key block kb visits the query blocks from kb on.  The heaviest (low kb) go
        // first over every (clip, head), so the last wave holds the lightest CTAs; key blocks
        // still start in ascending order, which the ordered dQ adds rely on.
        const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z), per = gridDim.y * gridDim.z;
        kb = lin / per;
        h = (lin % per) % gridDim.y;
        b = (lin % per) / gridDim.y;
    }
    const int k0 = kb * AB_BK;
    int kv_end = a.Tk;
    if (a.nvalid) kv_end = min(kv_end, a.nvalid[b]);
    const int nqb_all = (a.T + AB_BQ - 1) / AB_BQ;
    const int qb_first = k0 >= kv_end ? nqb_all : (a.causal ? k0 / AB_BQ : 0);
    const int nq = nqb_all - qb_first;  // query blocks this CTA visits

    if (threadIdx.x == 0) {
        mbar_init(kv_full, 1);
        mbar_init(s_full, 1);
        mbar_init(s_free, 8);   // one arrive per elementwise warp
        mbar_init(ds_full, 8);
        mbar_init(p_free, 1);
        mbar_init(ds_free(0), 1);
        mbar_init(ds_free(1), 1);
        mbar_init(dq_full, 1);
        mbar_init(dq_free, 4);
        mbar_init(acc_done, 1);
        for (int st = 0; st < AB_QD_STAGES; ++st) {
            mbar_init(qd_full(st), 1);
            mbar_init(qd_empty(st), 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(AB_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 320, tdQ = tmem + 384,
                   tP = tmem + 448;
    pdl_wait();
    pdl_trigger();

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ TMA producer
        if (nq > 0) {
            mbar_expect_tx(kv_full, 2 * AB_T16);
            tma_load_2d(base + AB_K_OFF, &maps.k, h * 64, b * a.Tk + k0, kv_full);
            tma_load_2d(base + AB_V_OFF, &maps.v, h * 64, b * a.Tk + k0, kv_full);
            for (int u = 0; u < nq; ++u) {
                const int st = u % AB_QD_STAGES, q0 = (qb_first + u) * AB_BQ;
                if (!mbar_wait(qd_empty(st), ((u / AB_QD_STAGES) & 1) ^ 1, err, 41)) break;
                const uint32_t dst = base + AB_QD_OFF + st * 2 * AB_T16;
                mbar_expect_tx(qd_full(st), 2 * AB_T16);
                tma_load_2d(dst, &maps.q, h * 64, b * a.T + q0, qd_full(st));
                tma_load_2d(dst + AB_T16, &maps.dout, h * 64, b * a.T + q0, qd_full(st));
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ MMA issuer
        constexpr uint32_t ID_S = IDESC_F16_F32ACC | (16u << 17) | (8u << 24);  // 128x128, K/K
        constexpr uint32_t ID_KV = IDESC_F16_F32ACC | (1u << 16) | (8u << 17) | (8u << 24);  // 128x64, K/MN
        constexpr uint32_t ID_Q = IDESC_F16_F32ACC | (1u << 15) | (1u << 16) | (8u << 17) |
                                  (8u << 24);  // 128x64, MN/MN
        const uint64_t dK_k = smem_desc(base + AB_K_OFF, 16, 1024), dV_k = smem_desc(base + AB_V_OFF, 16, 1024);
        const uint64_t dK_mn = smem_desc(base + AB_K_OFF, 8192, 1024);
        bool ok = nq > 0 && mbar_wait(kv_full, 0, err, 42);
        // S^T / dP^T of block u (reduction over d).  Block u + 1's are issued as soon as the
        // elementwise warps have read block u's out of TMEM, ahead of block u's dV / dK / dQ, so
        // the tensor core computes them while the P / dS pass of block u still runs.
        auto issue_s = [&](int u) {
            const uint32_t qs = base + AB_QD_OFF + (u % AB_QD_STAGES) * 2 * AB_T16;
            if (!mbar_wait(qd_full(u % AB_QD_STAGES), (u / AB_QD_STAGES) & 1, err, 43)) return false;
            if (u > 0 && !mbar_wait(s_free, (u - 1) & 1, err, 44)) return false;
            const uint64_t dQ_k = smem_desc(qs, 16, 1024), dO_k = smem_desc(qs + AB_T16, 16, 1024);
#pragma unroll
            for (int k16 = 0; k16 < 4; ++k16) {
                mma_f16(tS, dK_k + 2 * k16, dQ_k + 2 * k16, ID_S, k16 > 0 ? 1u : 0u);
                mma_f16(tdP, dV_k + 2 * k16, dO_k + 2 * k16, ID_S, k16 > 0 ? 1u : 0u);
            }
            mma_commit(s_full);
            return true;
        };
        if (ok) ok = issue_s(0);
        for (int u = 0; ok && u < nq; ++u) {
            const int st = u % AB_QD_STAGES;
            const uint32_t qs = base + AB_QD_OFF + st * 2 * AB_T16;
            if (u + 1 < nq && !issue_s(u + 1)) { ok = false; break; }
            const uint64_t dQ_mn = smem_desc(qs, 8192, 1024), dO_mn = smem_desc(qs + AB_T16, 8192, 1024);
            if (!mbar_wait(ds_full, u & 1, err, 45)) { ok = false; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");  // P^T stored by the pass
            const uint32_t dsb = base + AB_DS_OFF + (u & 1) * 2 * AB_T16;  // this block's dS^T buffer
            const uint64_t dS_k = smem_desc(dsb, 16, 1024), dS_mn = smem_desc(dsb, 16384, 1024);
            // dV first, so that P^T is released a third of the way through the block's MMAs
#pragma unroll
            for (int k16 = 0; k16 < 8; ++k16)  // dV += P^T dO   (reduction over queries; P^T in TMEM)
                mma_f16_ta(tdV, tP + 8 * k16, dO_mn + 128 * k16, ID_KV, (u > 0 || k16 > 0) ? 1u : 0u);
            mma_commit(p_free);
#pragma unroll
            for (int k16 = 0; k16 < 8; ++k16) {  // dK += dS^T Q
                const uint64_t ka = (uint64_t)((k16 >> 2) * (AB_T16 >> 4) + (k16 & 3) * 2);
                mma_f16(tdK, dS_k + ka, dQ_mn + 128 * k16, ID_KV, (u > 0 || k16 > 0) ? 1u : 0u);
            }
            if (u > 0 && !mbar_wait(dq_free, (u - 1) & 1, err, 46)) { ok = false; break; }
#pragma unroll
            for (int k16 = 0; k16 < 8; ++k16)  // dQ = dS K   (reduction over keys)
                mma_f16(tdQ, dS_mn + 128 * k16, dK_mn + 128 * k16, ID_Q, k16 > 0 ? 1u : 0u);
            mma_commit(ds_free(u & 1));
            mma_commit(qd_empty(st));
            mma_commit(dq_full);
        }
        if (ok && nq > 0) mma_commit(acc_done);
    } else if (warp >= 2 && warp < 10) {
        // ------------------------------------------------------------ P / dS, then dK / dV
        // two groups of four warps: group g takes query columns 64g .. 64g+63 of every block
        // (both groups read the same TMEM lanes), then group 0 writes dK and group 1 dV
        const int grp = (warp - 2) >> 2;
        const int quad = warp & 3;
        const int kr = quad * 32 + lane, key = k0 + kr;
        const uint32_t lb = (uint32_t)(quad * 32) << 16;
        const float sl2 = a.scale * AT_LOG2E;
        float* lsd = reinterpret_cast<float*>(smem + AB_LSE_OFF);
        unsigned char* dSt = smem + AB_DS_OFF;
        bool ok = true;
        // this thread's element of a block's lse (t < 64) or D (t >= 64), loaded one block ahead
        // so that the global-load latency overlaps the current block's work
        const int t = threadIdx.x - 64 - grp * 128, c = grp * 64 + (t & 63);
        auto fetch_ld = [&](int u) {
            const int qi = (qb_first + u) * AB_BQ + c;
            const long off = ((long)b * a.H + h) * a.T + qi;
            return (u < nq && qi < a.T) ? (t < 64 ? a.lse[off] : a.dvec[off]) : 0.f;
        };
        float next_ld = fetch_ld(0);
        for (int u = 0; u < nq; ++u) {
            const int q0 = (qb_first + u) * AB_BQ;
            {
                float* L = lsd + (u & 1) * 256;
                L[t < 64 ? c : 128 + c] = t < 64 ? -next_ld : next_ld;  // -lse | D
                if (grp == 0) asm volatile("bar.sync 1, 128;" ::: "memory");
                else asm volatile("bar.sync 3, 128;" ::: "memory");
            }
            next_ld = fetch_ld(u + 1);
            const float* L = lsd + (u & 1) * 256;
            // after a failed wait the loop keeps running (without work) so that every warp still
            // reaches each named barrier; waits after a failure return at once (error word set)
            if (ok) {
                if (lane == 0) ok = mbar_wait(s_full, u & 1, err, 47);
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            }
            if (!ok) continue;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            for (int qt = 2 * grp; qt < 2 * grp + 2; ++qt) {  // 32 query columns at a time
                float sv[32], dp[32];
                tmem_ld32_nw(tS + lb + qt * 32, sv);
                tmem_ld32_nw(tdP + lb + qt * 32, dp);
                tmem_wait_ld();
                if (qt == 2 * grp + 1) {  // this warp's S^T / dP^T consumed: the next block's may start
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) mbar_arrive(s_free);
                }
                const int qbase = q0 + qt * 32;
                // valid queries of this quarter for this key: q in [qlo, qhi)
                int qlo = 0, qhi = min(32, a.T - qbase);
                if (key >= kv_end) qhi = 0;
                if (a.causal) qlo = max(0, key - qbase);
                const float4* L4 = reinterpret_cast<const float4*>(L + qt * 32);         // -lse
                const float4* D4 = reinterpret_cast<const float4*>(L + 128 + qt * 32);   // D
                if (qlo == 0 && qhi == 32) {  // all but the edge blocks: pairs of columns
                    const float2 sl = make_float2(sl2, sl2);
#pragma unroll
                    for (int c4 = 0; c4 < 8; ++c4) {
                        const float4 l = L4[c4], dv = D4[c4];
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int c = 4 * c4 + 2 * e;
                            const float2 x = fma_f2(make_float2(sv[c], sv[c + 1]), sl,
                                                    e ? make_float2(l.z, l.w) : make_float2(l.x, l.y));
                            const float2 pv = make_float2(fast_ex2(x.x), fast_ex2(x.y));
                            const float2 ds = mul_f2(pv, sub_f2(make_float2(dp[c], dp[c + 1]),
                                                                e ? make_float2(dv.z, dv.w) : make_float2(dv.x, dv.y)));
                            sv[c] = pv.x; sv[c + 1] = pv.y;
                            dp[c] = ds.x; dp[c + 1] = ds.y;
                        }
                    }
                } else {
#pragma unroll
                    for (int c4 = 0; c4 < 8; ++c4) {
                        const float4 l = L4[c4], dv = D4[c4];
                        const float lv[4] = {l.x, l.y, l.z, l.w}, dd[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int c = 4 * c4 + e;
                            float pv = fast_ex2(fmaf(sv[c], sl2, lv[e]));
                            if (c < qlo || c >= qhi) pv = 0.f;
                            sv[c] = pv;
                            dp[c] = pv * (dp[c] - dd[e]);
                        }
                    }
                }
                if (qt == 2 * grp && u > 0) {
                    // P^T (TMEM): the previous block's dV MMAs have read it; dS^T buffer u & 1:
                    // block u - 2's dK / dQ MMAs have read it
                    if (lane == 0) {
                        ok = mbar_wait(p_free, (u - 1) & 1, err, 48);
                        if (ok && u > 1) ok = mbar_wait(ds_free(u & 1), ((u >> 1) - 1) & 1, err, 51);
                    }
                    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                    if (!ok) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                }
                {  // P^T of this key row, query columns qt*32 .. qt*32+31, as f16 pairs into TMEM
                    uint32_t pk[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) pk[j] = pack_f16(sv[2 * j], sv[2 * j + 1]);
                    tmem_st16(tP + lb + qt * 16, pk);
                }
#pragma unroll
                for (int un = 0; un < 4; ++un) {
                    const uint32_t off = (qt >> 1) * AB_T16 + at_sw128(kr, (qt & 1) * 4 + un);
                    *reinterpret_cast<uint4*>(dSt + (u & 1) * 2 * AB_T16 + off) =
                        make_uint4(pack_f16(dp[8 * un], dp[8 * un + 1]), pack_f16(dp[8 * un + 2], dp[8 * un + 3]),
                                   pack_f16(dp[8 * un + 4], dp[8 * un + 5]), pack_f16(dp[8 * un + 6], dp[8 * un + 7]));
                }
            }
            if (!ok) continue;
            tmem_wait_st();
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(ds_full);
        }
        // dK / dV epilogue
        bool have = ok && nq > 0;
        if (have) {
            if (lane == 0) have = mbar_wait(acc_done, 0, err, 49);
            have = __shfl_sync(0xffffffffu, have ? 1 : 0, 0) != 0;
        }
        if (have) asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int krow = min(key, a.Tk - 1);
        f16* dkr = a.dk + ((long)b * a.Tk + krow) * a.lddk + h * 64;
        f16* dvr = a.dv + ((long)b * a.Tk + krow) * a.lddv + h * 64;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
            float x[32];
            if (have) {
                tmem_ld32_nw((grp == 0 ? tdK : tdV) + lb + c * 32, x);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int e = 0; e < 32; ++e) x[e] = 0.f;
            }
            if (key < a.Tk) {
                if (grp == 0) {  // dK: scale, back to the unrotated frame, DoRA column factor
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        const int col = c * 32 + e;
                        float x0 = x[e] * a.scale, x1 = x[e + 1] * a.scale;
                        if (a.rope) {
                            const float2 t = reinterpret_cast<const float2*>(a.rope)[(long)key * 32 + col / 2];
                            const float y0 = x0 * t.x + x1 * t.y, y1 = -x0 * t.y + x1 * t.x;
                            x0 = y0;
                            x1 = y1;
                        }
                        if (a.kscale) {
                            x0 *= a.kscale[h * 64 + col];
                            x1 *= a.kscale[h * 64 + col + 1];
                        }
                        x[e] = x0;
                        x[e + 1] = x1;
                    }
                } else if (a.vscale) {  // dV: DoRA column factor
#pragma unroll
                    for (int e = 0; e < 32; ++e) x[e] *= a.vscale[h * 64 + c * 32 + e];
                }
                f16* dst = (grp == 0 ? dkr : dvr) + c * 32;
#pragma unroll
                for (int un = 0; un < 4; ++un)
                    *reinterpret_cast<uint4*>(dst + 8 * un) =
                        make_uint4(pack_f16(x[8 * un], x[8 * un + 1]), pack_f16(x[8 * un + 2], x[8 * un + 3]),
                                   pack_f16(x[8 * un + 4], x[8 * un + 5]), pack_f16(x[8 * un + 6], x[8 * un + 7]));
            }
        }
    } else if (warp >= 10) {
        // ------------------------------------------------------------ dQ epilogue (reduce-add)
        const int quad = warp & 3;
        const int qr = quad * 32 + lane;
        const uint32_t lb = (uint32_t)(quad * 32) << 16;
        unsigned char* stg = smem + AB_DQ_OFF;
        const bool leader = threadIdx.x == 320;
        bool ok = true;
        for (int u = 0; u < nq; ++u) {
            const int q0 = (qb_first + u) * AB_BQ;
            // as above: a failed wait skips the work but not the named barriers
            if (ok) {
                if (lane == 0) ok = mbar_wait(dq_full, u & 1, err, 50);
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            }
            float d[64];
            if (ok) {
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                tmem_ld32_nw(tdQ + lb, d);
                tmem_ld32_nw(tdQ + lb + 32, d + 32);
                tmem_wait_ld();
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(dq_free);
            } else {
#pragma unroll
                for (int e = 0; e < 64; ++e) d[e] = 0.f;
            }
            // ordered adds: this key block's turn comes after the earlier key blocks that add to
            // this query block (key blocks 0 .. kb contribute, in that order); bounded wait
            int* turn = a.dq_turn ? a.dq_turn + ((long)b * a.H + h) * nqb_all + (qb_first + u) : nullptr;
            // (a wait that gives up has recorded its code: the step fails; the add still goes, so
            // the later key blocks are not held up)
            if (turn && leader) (void)flag_wait(turn, kb, err, 52);
            // one 32-column half at a time through the single staging tile
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                // the previous reduce has finished reading the staging tile
                if (leader) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                asm volatile("bar.sync 2, 128;" ::: "memory");
#pragma unroll
                for (int un = 0; un < 8; ++un) {
                    const float* x = d + half * 32 + 4 * un;
                    *reinterpret_cast<float4*>(stg + at_sw128(qr, un)) =
                        make_float4(x[0] * a.scale, x[1] * a.scale, x[2] * a.scale, x[3] * a.scale);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                asm volatile("bar.sync 2, 128;" ::: "memory");
                if (leader) {
                    asm volatile(
                        "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%1, %2}], [%3];"
                        ::"l"(reinterpret_cast<uint64_t>(&maps.dq)), "r"(h * 64 + half * 32), "r"(b * a.T + q0),
                          "r"(base + AB_DQ_OFF)
                        : "memory");
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
            }
            if (turn && leader) {
                // this block's adds are performed before the next key block may add
                asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
                asm volatile("fence.proxy.async.global;" ::: "memory");
                red_release_add(turn, 1);
            }
        }
        if (leader) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // staging read
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(AB_TMEM_COLS));
}

// fp32 tensor map for the dQ reduce: [rows][ld] fp32, box 32 x 128, 128-byte swizzle
void make_f32_map(CUtensorMap* map, const float* ptr, long rows, long cols, long ld) {
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (ld * 4) % 16) throw std::runtime_error("attn_bwd_tc: dq_acc alignment");
    typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static EncodeFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !p)
            throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
        fn = reinterpret_cast<EncodeFn>(p);
    }
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
    cuuint32_t box[2] = {32, 128};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (dq) failed: " + std::to_string((int)r));
}

}  // namespace

bool attn_fwd_tc_supported(const AttnArgs& a) {
    if (a.rope_load || a.H <= 0 || a.T <= 0 || a.clips <= 0 || a.Tk < AT_BK) return false;
    if ((a.ldq * 2) % 16 || (a.ldk * 2) % 16 || (a.ldv * 2) % 16 || (a.ldo % 8)) return false;
    const uintptr_t al = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                         reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.o);
    return (al & 15) == 0;
}

void attn_fwd_tc(const AttnArgs& a, int* err, cudaStream_t s) {
    if (!attn_fwd_tc_supported(a)) throw std::runtime_error("attn_fwd_tc: unsupported arguments");
    AtMaps maps;
    // token-major [clips * T][ld] tensors; a box is 64 columns (one head) x 128 rows
    tc_make_map(&maps.q, a.q, (long)a.clips * a.T, (long)a.H * AT_HD, a.ldq, AT_HD, AT_BQ);
    tc_make_map(&maps.k, a.k, (long)a.clips * a.Tk, (long)a.H * AT_HD, a.ldk, AT_HD, AT_BK);  // 64 x 64
    tc_make_map(&maps.v, a.v, (long)a.clips * a.Tk, (long)a.H * AT_HD, a.ldv, AT_HD, AT_BK);
    static DeviceOnce once;
    once([] { cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM); });
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((a.T + AT_BQ - 1) / AT_BQ, a.H, a.clips);
        cfg.blockDim = dim3(AT_THREADS, 1, 1);
        cfg.dynamicSmemBytes = AT_SMEM;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        pdl_attr(attr[0]);
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaLaunchKernelEx(&cfg, attn_fwd_tc_kernel, maps, a, err);
    }
}

}  // namespace act

namespace act {

bool attn_bwd_tc_supported(const AttnArgs& a) {
    if (!attn_fwd_tc_supported(a) || !a.dout || !a.dq_acc || !a.dk || !a.dv || !a.dvec) return false;
    if ((a.lddo * 2) % 16 || (a.ldq_acc * 4) % 16 || (a.lddk % 8) || (a.lddv % 8)) return false;
    const uintptr_t al = reinterpret_cast<uintptr_t>(a.dout) | reinterpret_cast<uintptr_t>(a.dq_acc) |
                         reinterpret_cast<uintptr_t>(a.dk) | reinterpret_cast<uintptr_t>(a.dv);
    return (al & 15) == 0 && a.Tk >= AB_BK;
}

void attn_bwd_tc(const AttnArgs& a, int* err, cudaStream_t s) {
    if (!attn_bwd_tc_supported(a)) throw std::runtime_error("attn_bwd_tc: unsupported arguments");
    attn_dvec(a, s);
    AbMaps maps;
    tc_make_map(&maps.q, a.q, (long)a.clips * a.T, (long)a.H * 64, a.ldq, 64, AB_BQ);
    tc_make_map(&maps.dout, a.dout, (long)a.clips * a.T, (long)a.H * 64, a.lddo, 64, AB_BQ);
    tc_make_map(&maps.k, a.k, (long)a.clips * a.Tk, (long)a.H * 64, a.ldk, 64, AB_BK);
    tc_make_map(&maps.v, a.v, (long)a.clips * a.Tk, (long)a.H * 64, a.ldv, 64, AB_BK);
    make_f32_map(&maps.dq, a.dq_acc, (long)a.clips * a.T, (long)a.H * 64, a.ldq_acc);
    static DeviceOnce once;
    once([] { cudaFuncSetAttribute(attn_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AB_SMEM); });
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((a.Tk + AB_BK - 1) / AB_BK, a.H, a.clips);
        cfg.blockDim = dim3(AB_THREADS, 1, 1);
        cfg.dynamicSmemBytes = AB_SMEM;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        pdl_attr(attr[0]);
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaLaunchKernelEx(&cfg, attn_bwd_tc_kernel, maps, a, err);
    }
}

}  // namespace act
