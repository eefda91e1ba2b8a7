// xattn_tc.cu -- cross-attention over few keys (at most 64 per clip) on the tcgen05 tensor cores,
// head_dim 64.
//
// The conditioning attention of src/ac/transformer.h:108-125: softmax(scale K^T Q + mask) V with
// the optional implicit zero key (score 0, value 0: src/ac/transformer.h:74-79) and per-clip
// valid-key counts (the -inf columns past valid_tokens, src/mf/train.h:169-175).  With every key
// of a clip inside one 64-key block a query row's softmax is complete in one pass, so both
// kernels are query-major -- one CTA per 128 queries of one (clip, head) -- and the backward
// needs neither the forward's log-sum-exp nor rowsum(dO * O):
//
// Forward:  S = Q K^T (128 x 64, fp32 in TMEM); one query row per thread: the exact softmax over
//           the valid keys and the zero key, P as f16 pairs written over S's TMEM columns;
//           O = P V (P read from TMEM, V MN-major); O (f16) and the base-2 LSE out.
// Backward: S = Q K^T and dP = dO V^T (TMEM); the softmax recomputed row by row;
//           D = sum_j P_j dP_j (rowsum(dO * O) without reading O: O = sum_j P_j V_j);
//           dS = P (dP - D) to shared memory (queries x keys, 128-byte swizzle);
//           dQ = scale dS K (f16, times the optional DoRA column factor, straight to the output);
//           with an adapter on the conditioning's K / V: dV = P^T dO and dK = scale dS^T Q for
//           this block's 128 queries into an fp32 slice per query block, which attn_dkv_finish
//           adds in block order (the same sum whichever CTA finishes first).  P^T and dS^T are
//           the shared tiles read as MN-major A operands; M = 128 rows are issued, of which
//           the keys 64..127 read the next tile in shared memory and are never stored.
//
// Q / dO / K / V come in through 3-D tensor maps [clips][rows][cols], so rows past a clip's
// queries or stored keys read as zero (no clip sees its neighbour's rows); keys past the valid
// count are masked in the row pass.  Warp 0 lane 0 issues the TMA loads and the MMAs; warps 1..4
// are the row pass (warp w reads TMEM lanes 32 (w % 4) ..).  Every mbarrier wait is bounded and
// reports into the error word; TMEM is released on every path.
#include <cuda.h>

#include <stdexcept>
#include <string>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace act {

namespace {

using namespace tc;

constexpr int XA_BQ = 128;                   // queries per CTA
constexpr int XA_BK = 64;                    // keys (all of a clip's)
constexpr int XA_QT = XA_BQ * 64 * 2;        // 16 KB: 128 rows x 64 f16
constexpr int XA_KT = XA_BK * 64 * 2;        //  8 KB: 64 rows x 64 f16
constexpr int XA_THREADS = 5 * 32;
constexpr float XA_LOG2E = 1.4426950408889634f;

// forward shared memory: Q | K | V | barriers
constexpr int XF_Q = 0, XF_K = XA_QT, XF_V = XF_K + XA_KT, XF_BAR = XF_V + XA_KT;
constexpr int XF_SMEM = XF_BAR + 64 + 1024;
constexpr uint32_t XF_TMEM = 128;            // S, then P (f16 pairs): 0..63;  O: 64..127

// backward shared memory: Q | dO | [P] | dS | K | V | barriers.  P and dS are each followed by
// a 16 KB region (dS, K + V), which the M = 128 MN-major reads of dV / dK reach for keys 64..127.
template <bool DKV>
struct XbLayout {
    static constexpr int Q = 0, DO = XA_QT;
    static constexpr int P = 2 * XA_QT;      // only with DKV
    static constexpr int DS = DKV ? 3 * XA_QT : 2 * XA_QT;
    static constexpr int K = DS + XA_QT, V = K + XA_KT, BAR = V + XA_KT;
    static constexpr int SMEM = BAR + 64 + 1024;
    static constexpr uint32_t TMEM = DKV ? 256 : 128;  // S 0..63, dP then dQ 64..127, dV 128..191, dK 192..255
};

struct XaMaps {
    CUtensorMap q, k, v, dout;
};

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void ld32(uint32_t taddr, float* f) {
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

__device__ __forceinline__ void ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void st32(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// D (+)= A B with A in tensor memory (lane = row, two f16 K elements per 32-bit column)
__device__ __forceinline__ void mma_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 128 x 64 accumulators: M = 128 (bits 24..28 = M >> 4), N = 64 (bits 17..22 = N >> 3);
// bit 15 / 16: A / B MN-major
constexpr uint32_t XA_ID = IDESC_F16_F32ACC | ((uint32_t)(64 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
constexpr uint32_t XA_ID_KK = XA_ID;                            // A K-major, B K-major
constexpr uint32_t XA_ID_KM = XA_ID | (1u << 16);               // A K-major, B MN-major
constexpr uint32_t XA_ID_MM = XA_ID | (1u << 15) | (1u << 16);  // both MN-major

// The row pass's softmax of one query row over the 64 key columns s[] (raw scores): keys at or
// past kv_end masked, the zero key optional.  On return s[] holds the probabilities; m2 is the
// base-2 maximum used (0 when nothing is in range) and l the sum of exponentials.
__device__ __forceinline__ void row_softmax(float* s, int kv_end, float sl2, bool zero_key, float& m2, float& l) {
#pragma unroll
    for (int c = 0; c < XA_BK; ++c)
        if (c >= kv_end) s[c] = -INFINITY;
    float mx[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) mx[e] = s[e];
#pragma unroll
    for (int c = 8; c < XA_BK; ++c) mx[c & 7] = fmaxf(mx[c & 7], s[c]);
    const float mb = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                           fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * sl2;
    const float m = zero_key ? fmaxf(mb, 0.f) : mb;
    m2 = m == -INFINITY ? 0.f : m;
    float sum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < XA_BK; ++c) {
        s[c] = ex2(fmaf(s[c], sl2, -m2));  // masked: ex2(-inf) = 0
        sum[c & 3] += s[c];
    }
    l = (sum[0] + sum[1]) + (sum[2] + sum[3]);
    if (zero_key) l += ex2(-m2);
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int c = 0; c < XA_BK; ++c) s[c] *= inv;
}

// 32 f16 values (columns 32 half .. +31 of row r) into a 128-byte-swizzled [rows][64] tile
__device__ __forceinline__ void store_half_sw128(unsigned char* tile, int r, int half, const float* x) {
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        const int u = 4 * half + v;
        *reinterpret_cast<uint4*>(tile + r * 128 + ((u ^ (r & 7)) << 4)) =
            make_uint4(pack_f16(x[8 * v], x[8 * v + 1]), pack_f16(x[8 * v + 2], x[8 * v + 3]),
                       pack_f16(x[8 * v + 4], x[8 * v + 5]), pack_f16(x[8 * v + 6], x[8 * v + 7]));
    }
}

__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

// ---------------------------------------------------------------------------------------
// forward

__global__ void __launch_bounds__(XA_THREADS, 4) xattn_fwd_tc_kernel(const __grid_constant__ XaMaps maps,
                                                                     const AttnArgs a, int* err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023) & ~1023u;
    unsigned char* smem = smem_raw + (base - raw);
    const uint32_t bars = base + XF_BAR;
    const uint32_t in_full = bars, s_full = bars + 8, p_full = bars + 16, o_full = bars + 24;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + XF_BAR + 32);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int q0 = qb * XA_BQ;

    if (threadIdx.x == 0) {
        prefetch_tmap(&maps.q);
        prefetch_tmap(&maps.k);
        prefetch_tmap(&maps.v);
        mbar_init(in_full, 1);
        mbar_init(s_full, 1);
        mbar_init(p_full, 4);  // one arrive per row-pass warp
        mbar_init(o_full, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) tmem_alloc(smem_u32(tmem_slot), XF_TMEM);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS = tmem, tO = tmem + 64;
    pdl_wait();
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            mbar_expect_tx(in_full, XA_QT + 2 * XA_KT);
            tma_load_3d(base + XF_Q, &maps.q, h * 64, q0, b, in_full);
            tma_load_3d(base + XF_K, &maps.k, h * 64, 0, b, in_full);
            tma_load_3d(base + XF_V, &maps.v, h * 64, 0, b, in_full);
            const uint64_t dq = smem_desc(base + XF_Q, 16, 1024), dk = smem_desc(base + XF_K, 16, 1024);
            const uint64_t dv = smem_desc(base + XF_V, 8192, 1024);
            uint32_t last = 0, last_par = 0;  // the last barrier a commit of this thread arrives on
            if (mbar_wait(in_full, 0, err, 71)) {
#pragma unroll
                for (int k16 = 0; k16 < 4; ++k16)  // S = Q K^T (reduction over d)
                    mma_f16(tS, dq + 2 * k16, dk + 2 * k16, XA_ID_KK, k16 > 0 ? 1u : 0u);
                mma_commit(s_full);
                last = s_full;
                if (mbar_wait(p_full, 0, err, 72)) {
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                    for (int k16 = 0; k16 < 4; ++k16)  // O = P V: P in TMEM (8 columns per 16 keys), V MN-major
                        mma_ta(tO, tS + 8 * k16, dv + 128 * k16, XA_ID_KM, k16 > 0 ? 1u : 0u);
                    mma_commit(o_full);
                    last = o_full;
                }
            } else {
                mbar_wait_drain(in_full, 0);  // the loads still land before the CTA exits
            }
            if (last) mbar_wait_drain(last, last_par);  // no MMA in flight when TMEM is released
        }
    } else {
        // ------------------------------------------------------------ row pass
        const int quad = warp & 3;
        const int r = quad * 32 + lane, i = q0 + r;
        const uint32_t lb = (uint32_t)(quad * 32) << 16;
        int kv_end = min(a.Tk, XA_BK);
        if (a.nvalid) kv_end = min(kv_end, a.nvalid[b]);
        bool ok = true;
        if (lane == 0) ok = mbar_wait(s_full, 0, err, 73);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        float m2 = 0.f, l = 0.f;
        if (ok) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            float s[XA_BK];
            ld32(tS + lb, s);
            ld32(tS + lb + 32, s + 32);
            ld_wait();
            row_softmax(s, kv_end, a.scale * XA_LOG2E, a.zero_key != 0, m2, l);
            uint32_t pk[32];
#pragma unroll
            for (int c2 = 0; c2 < 32; ++c2) pk[c2] = pack_f16(s[2 * c2], s[2 * c2 + 1]);
            st32(tS + lb, pk);  // over S's first 32 columns: the A operand of O = P V
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        bool have_o = ok;
        if (have_o) {
            if (lane == 0) have_o = mbar_wait(o_full, 0, err, 74);
            have_o = __shfl_sync(0xffffffffu, have_o ? 1 : 0, 0) != 0;
        }
        if (have_o) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            float o[64];
            ld32(tO + lb, o);
            ld32(tO + lb + 32, o + 32);
            ld_wait();
            if (i < a.T) {
                f16* orow = a.o + ((long)b * a.T + i) * a.ldo + h * 64;
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    *reinterpret_cast<uint4*>(orow + 8 * u) =
                        make_uint4(pack_f16(o[8 * u], o[8 * u + 1]), pack_f16(o[8 * u + 2], o[8 * u + 3]),
                                   pack_f16(o[8 * u + 4], o[8 * u + 5]), pack_f16(o[8 * u + 6], o[8 * u + 7]));
                if (a.lse) a.lse[((long)b * a.H + h) * a.T + i] = m2 + __log2f(l);
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(XF_TMEM));
}

// ---------------------------------------------------------------------------------------
// backward

template <bool DKV>
__global__ void __launch_bounds__(XA_THREADS, DKV ? 2 : 3) xattn_bwd_tc_kernel(const __grid_constant__ XaMaps maps,
                                                                              const AttnArgs a, int* err) {
    using L = XbLayout<DKV>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023) & ~1023u;
    unsigned char* smem = smem_raw + (base - raw);
    const uint32_t bars = base + L::BAR;
    const uint32_t in_full = bars, s_full = bars + 8, ds_full = bars + 16, acc_full = bars + 24;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR + 32);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int q0 = qb * XA_BQ;

    if (threadIdx.x == 0) {
        prefetch_tmap(&maps.q);
        prefetch_tmap(&maps.k);
        prefetch_tmap(&maps.v);
        prefetch_tmap(&maps.dout);
        mbar_init(in_full, 1);
        mbar_init(s_full, 1);
        mbar_init(ds_full, 4);
        mbar_init(acc_full, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) tmem_alloc(smem_u32(tmem_slot), L::TMEM);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS = tmem, tdP = tmem + 64, tdQ = tmem + 64, tdV = tmem + 128, tdK = tmem + 192;
    pdl_wait();
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            mbar_expect_tx(in_full, 2 * XA_QT + 2 * XA_KT);
            tma_load_3d(base + L::Q, &maps.q, h * 64, q0, b, in_full);
            tma_load_3d(base + L::DO, &maps.dout, h * 64, q0, b, in_full);
            tma_load_3d(base + L::K, &maps.k, h * 64, 0, b, in_full);
            tma_load_3d(base + L::V, &maps.v, h * 64, 0, b, in_full);
            const uint64_t q_k = smem_desc(base + L::Q, 16, 1024), do_k = smem_desc(base + L::DO, 16, 1024);
            const uint64_t k_k = smem_desc(base + L::K, 16, 1024), v_k = smem_desc(base + L::V, 16, 1024);
            const uint64_t k_mn = smem_desc(base + L::K, 8192, 1024);
            const uint64_t ds_k = smem_desc(base + L::DS, 16, 1024);
            uint32_t last = 0;
            if (mbar_wait(in_full, 0, err, 75)) {
#pragma unroll
                for (int k16 = 0; k16 < 4; ++k16) {  // S = Q K^T, dP = dO V^T (reduction over d)
                    mma_f16(tS, q_k + 2 * k16, k_k + 2 * k16, XA_ID_KK, k16 > 0 ? 1u : 0u);
                    mma_f16(tdP, do_k + 2 * k16, v_k + 2 * k16, XA_ID_KK, k16 > 0 ? 1u : 0u);
                }
                mma_commit(s_full);
                last = s_full;
                if (mbar_wait(ds_full, 0, err, 76)) {
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                    for (int k16 = 0; k16 < 4; ++k16)  // dQ = dS K (reduction over keys; K MN-major)
                        mma_f16(tdQ, ds_k + 2 * k16, k_mn + 128 * k16, XA_ID_KM, k16 > 0 ? 1u : 0u);
                    if (DKV) {
                        // P^T / dS^T: the [queries][keys] tiles as MN-major A (M = keys), 16 queries per step
                        const uint64_t p_mn = smem_desc(base + L::P, 16384, 1024);
                        const uint64_t ds_mn = smem_desc(base + L::DS, 16384, 1024);
                        const uint64_t do_mn = smem_desc(base + L::DO, 8192, 1024);
                        const uint64_t q_mn = smem_desc(base + L::Q, 8192, 1024);
#pragma unroll
                        for (int k16 = 0; k16 < 8; ++k16) {  // dV = P^T dO, dK = dS^T Q (reduction over queries)
                            mma_f16(tdV, p_mn + 128 * k16, do_mn + 128 * k16, XA_ID_MM, k16 > 0 ? 1u : 0u);
                            mma_f16(tdK, ds_mn + 128 * k16, q_mn + 128 * k16, XA_ID_MM, k16 > 0 ? 1u : 0u);
                        }
                    }
                    mma_commit(acc_full);
                    last = acc_full;
                }
            } else {
                mbar_wait_drain(in_full, 0);
            }
            if (last) mbar_wait_drain(last, 0);
        }
    } else {
        // ------------------------------------------------------------ row pass
        const int quad = warp & 3;
        const int r = quad * 32 + lane, i = q0 + r;
        const uint32_t lb = (uint32_t)(quad * 32) << 16;
        int kv_end = min(a.Tk, XA_BK);
        if (a.nvalid) kv_end = min(kv_end, a.nvalid[b]);
        bool ok = true;
        if (lane == 0) ok = mbar_wait(s_full, 0, err, 77);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (ok) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            float s[XA_BK];
            ld32(tS + lb, s);
            ld32(tS + lb + 32, s + 32);
            ld_wait();
            float m2, l;
            row_softmax(s, kv_end, a.scale * XA_LOG2E, a.zero_key != 0, m2, l);
            if (i >= a.T)  // rows past the clip add nothing to dK / dV
#pragma unroll
                for (int c = 0; c < XA_BK; ++c) s[c] = 0.f;
            if (DKV) {
                store_half_sw128(smem + L::P, r, 0, s);
                store_half_sw128(smem + L::P, r, 1, s + 32);
            }
            // D = sum_j P_j dP_j (the zero key's dP is 0); dP is read from TMEM twice, 32 columns
            // at a time, to keep the register footprint at one row of P plus half a row
            float dp[32];
            float dsum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                ld32(tdP + lb + 32 * half, dp);
                ld_wait();
#pragma unroll
                for (int c = 0; c < 32; ++c) dsum[c & 3] = fmaf(s[32 * half + c], dp[c], dsum[c & 3]);
            }
            const float D = (dsum[0] + dsum[1]) + (dsum[2] + dsum[3]);
#pragma unroll
            for (int half = 0; half < 2; ++half) {  // dS = P (dP - D)
                ld32(tdP + lb + 32 * half, dp);
                ld_wait();
#pragma unroll
                for (int c = 0; c < 32; ++c) dp[c] = s[32 * half + c] * (dp[c] - D);
                store_half_sw128(smem + L::DS, r, half, dp);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor core
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(ds_full);
        bool have = ok;
        if (have) {
            if (lane == 0) have = mbar_wait(acc_full, 0, err, 78);
            have = __shfl_sync(0xffffffffu, have ? 1 : 0, 0) != 0;
        }
        if (have) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            {  // dQ row, 32 columns at a time
                f16* dst = a.dq_h + ((long)b * a.T + min(i, a.T - 1)) * a.lddq_h + h * 64;
                const float* cs = a.dq_scale ? a.dq_scale + h * 64 : nullptr;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float x[32];
                    ld32(tdQ + lb + 32 * half, x);  // warp-collective: every lane takes part
                    ld_wait();
                    if (i < a.T)
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            const int c0 = 32 * half + 8 * v;
                            float y[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) y[e] = x[8 * v + e] * a.scale * (cs ? cs[c0 + e] : 1.f);
                            *reinterpret_cast<uint4*>(dst + c0) = make_uint4(
                                pack_f16(y[0], y[1]), pack_f16(y[2], y[3]), pack_f16(y[4], y[5]), pack_f16(y[6], y[7]));
                        }
                }
            }
            if (DKV && quad < 2) {  // TMEM lanes 0..63: one key row per thread, this block's share in fp32
                const int j = quad * 32 + lane;
                const long at = (((long)qb * a.clips + b) * a.Tk + min(j, a.Tk - 1)) * a.H * 64 + h * 64;
#pragma unroll
                for (int which = 0; which < 2; ++which) {  // dK (times scale), then dV
                    const float* cs = which ? a.vscale : a.kscale;
                    const float f = which ? 1.f : a.scale;
                    float* dst = (which ? a.dv_acc : a.dk_acc) + at;
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        float x[32];
                        ld32((which ? tdV : tdK) + lb + 32 * half, x);
                        ld_wait();
                        if (j < a.Tk)
#pragma unroll
                            for (int c = 0; c < 32; c += 4) {
                                const int cc = 32 * half + c;
                                float4 y;
                                y.x = x[c] * f * (cs ? cs[h * 64 + cc] : 1.f);
                                y.y = x[c + 1] * f * (cs ? cs[h * 64 + cc + 1] : 1.f);
                                y.z = x[c + 2] * f * (cs ? cs[h * 64 + cc + 2] : 1.f);
                                y.w = x[c + 3] * f * (cs ? cs[h * 64 + cc + 3] : 1.f);
                                *reinterpret_cast<float4*>(dst + cc) = y;
                            }
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::TMEM));
}

template <class K>
void launch_xattn(K kern, const XaMaps& maps, const AttnArgs& a, int* err, int smem, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.T + XA_BQ - 1) / XA_BQ, a.H, a.clips);
    cfg.blockDim = dim3(XA_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    pdl_attr(attr[0]);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, maps, a, err);
}

}  // namespace

bool xattn_tc_supported(const AttnArgs& a) {
    if (a.causal || a.rope || a.rope_load || a.H <= 0 || a.T <= 0 || a.clips <= 0 || a.Tk <= 0 || a.Tk > XA_BK)
        return false;
    if ((a.ldq * 2) % 16 || (a.ldk * 2) % 16 || (a.ldv * 2) % 16 || a.ldo % 8) return false;
    const uintptr_t al = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                         reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.o);
    return (al & 15) == 0;
}

bool xattn_bwd_tc_supported(const AttnArgs& a) {
    if (!xattn_tc_supported(a) || !a.dout || !a.dq_h || (a.lddo * 2) % 16 || a.lddq_h % 8) return false;
    if ((reinterpret_cast<uintptr_t>(a.dout) | reinterpret_cast<uintptr_t>(a.dq_h)) & 15) return false;
    if (a.dk_acc || a.dv_acc) {  // dK / dV: one fp32 slice per query block, finished by attn_dkv_finish
        if (!a.dk_acc || !a.dv_acc || !a.dk || !a.dv || a.qsplit != (a.T + XA_BQ - 1) / XA_BQ) return false;
        if ((reinterpret_cast<uintptr_t>(a.dk_acc) | reinterpret_cast<uintptr_t>(a.dv_acc)) & 15) return false;
    }
    return true;
}

void xattn_fwd_tc(const AttnArgs& a, int* err, cudaStream_t s) {
    if (!xattn_tc_supported(a)) throw std::runtime_error("xattn_fwd_tc: unsupported arguments");
    XaMaps maps;
    tc_make_map3(&maps.q, a.q, a.clips, a.T, (long)a.H * 64, a.ldq, 64, XA_BQ);
    tc_make_map3(&maps.k, a.k, a.clips, a.Tk, (long)a.H * 64, a.ldk, 64, XA_BK);
    tc_make_map3(&maps.v, a.v, a.clips, a.Tk, (long)a.H * 64, a.ldv, 64, XA_BK);
    maps.dout = maps.q;
    static DeviceOnce once;
    once([] { cudaFuncSetAttribute(xattn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, XF_SMEM); });
    launch_xattn(xattn_fwd_tc_kernel, maps, a, err, XF_SMEM, s);
}

void xattn_bwd_tc(const AttnArgs& a, int* err, cudaStream_t s) {
    if (!xattn_bwd_tc_supported(a)) throw std::runtime_error("xattn_bwd_tc: unsupported arguments");
    XaMaps maps;
    tc_make_map3(&maps.q, a.q, a.clips, a.T, (long)a.H * 64, a.ldq, 64, XA_BQ);
    tc_make_map3(&maps.dout, a.dout, a.clips, a.T, (long)a.H * 64, a.lddo, 64, XA_BQ);
    tc_make_map3(&maps.k, a.k, a.clips, a.Tk, (long)a.H * 64, a.ldk, 64, XA_BK);
    tc_make_map3(&maps.v, a.v, a.clips, a.Tk, (long)a.H * 64, a.ldv, 64, XA_BK);
    static DeviceOnce once;
    once([] {
        cudaFuncSetAttribute(xattn_bwd_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             XbLayout<false>::SMEM);
        cudaFuncSetAttribute(xattn_bwd_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             XbLayout<true>::SMEM);
    });
    if (a.dk_acc) {
        launch_xattn(xattn_bwd_tc_kernel<true>, maps, a, err, XbLayout<true>::SMEM, s);
        attn_dkv_finish(a, s);
    } else {
        launch_xattn(xattn_bwd_tc_kernel<false>, maps, a, err, XbLayout<false>::SMEM, s);
    }
}

}  // namespace act
