// gemm_skinny.cu -- the LoRA rank-block products on the tcgen05 tensor cores.
//
// Every adapted projection adds four products whose small side is the rank block (RP <= 64
// columns) and whose large side is a whole activation / gradient matrix, read once:
//   U  = s X A^T         rows x RP,  reduction over in     (A = X K-major,   B = A_h K-major)
//   dU = s dY B          rows x RP,  reduction over out    (A = dY K-major,  B = B_h MN-major)
//   dB += dY^T U         out  x RP,  reduction over rows   (A = dY MN-major, B = U MN-major)
//   dA += (dU^T X)       stored transposed [RP][in]; the tile is in x RP, reduction over rows
// (src/ac/lora.h:34-95 and src/mf/train.h:150-190 for the products; the reference runs them as
// separate ggml mul_mat nodes).  They are HBM-bound: the kernel's job is to stream the large
// operand at full bandwidth.  Each CTA owns one 128-row tile and one slice of the reduction
// (split-K), so a few hundred CTAs keep enough bytes in flight; TMA stages 128 x 64 and 64 x 64
// boxes (128-byte swizzle, out-of-range rows and columns read as zero), one thread issues
// tcgen05.mma 128 x 64 x 16 into TMEM, and four epilogue warps finish the tile:
//   ACC      fp32, added into the gradient (row-major)
//   ACC_T    fp32, added into the gradient, transposed (tile rows are the gradient's columns)
//   STORE    f16 result.
// The split-K CTAs of a tile form one thread-block cluster; each leaves its fp32 partial tile in
// its own shared memory and, after a cluster barrier, reduces its share of the rows over all
// partials through distributed shared memory in split order, then converts and stores (STORE) or
// adds the sum into the gradient with one read-modify-write (ACC kinds: the cluster owns those
// entries in this launch).  No atomics: the result does not depend on the order in which CTAs
// finish, so a step (and a resumed run) is bit-for-bit reproducible.
// The large operand may also be a frozen weight kept as Q8_0 blocks (the DoRA products P = W A^T
// and BD^T W): the producer then brings each k-block's raw quants and scales into a slot beside
// the stage, and four converter warps write the f16 A tile in the swizzled layout the MMA reads
// (the same conversion as the projection GEMM's), so the weight is never expanded in memory.
// Every mbarrier wait is bounded (the shared error word records the site).
#include <cuda.h>

#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace act {

namespace {

using namespace tc;

constexpr int SK_BM = 128;
constexpr int SK_BN = 64;
constexpr int SK_BK = 64;
constexpr int SK_STAGES = 4;
constexpr int SK_A_BYTES = SK_BM * SK_BK * 2;  // 16 KB
constexpr int SK_B_BYTES = SK_BN * SK_BK * 2;  //  8 KB
constexpr int SK_STAGE = SK_A_BYTES + SK_B_BYTES;
constexpr int SK_SMEM = SK_STAGES * SK_STAGE + 1024 /*align*/ + 128 /*barriers, TMEM slot, flag*/;
constexpr int SK_THREADS = 6 * 32;
// Q8_0 A: per stage a raw slot of 128 x 64 quants and their 256 scales; four converter warps
constexpr int SK_RAW_Q = SK_BM * SK_BK;
constexpr int SK_RAW = (SK_RAW_Q + 2 * SK_BM * 2 + 1023) / 1024 * 1024;
constexpr int SK_SMEM_Q8 = SK_STAGES * (SK_STAGE + SK_RAW) + 1024 + 128;
constexpr int SK_THREADS_Q8 = 10 * 32;

struct SkParams {
    int M, K, nb;          // output tile rows, reduction length, valid columns (<= 64)
    int a_mn, b_mn;        // operand majorness
    int kind;              // SKINNY_ACC / SKINNY_ACC_T / SKINNY_STORE
    float alpha;
    void* out;
    long ldo;
    int splits;            // STORE with splits > 1: the cluster size along y
    int* err;
};

struct SkMaps {
    CUtensorMap a, b;
    CUtensorMap as;  // Q8_0 A: the block scales (a then maps the quants)
};

constexpr int SK_PART_LD = SK_BN + 4;  // partial-tile row stride (floats): conflict-free float4 rows

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t map_cta(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

template <bool Q8A>
__global__ void __launch_bounds__(Q8A ? SK_THREADS_Q8 : SK_THREADS, Q8A ? 1 : 2)
    skinny_kernel(const __grid_constant__ SkMaps maps, const SkParams p) {
    constexpr int NT = Q8A ? SK_THREADS_Q8 : SK_THREADS;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023) & ~1023u;
    unsigned char* smem = smem_raw + (base - raw);
    constexpr uint32_t RAW_OFF = SK_STAGES * SK_STAGE;                    // Q8A: raw slots
    constexpr uint32_t BAR_OFF = RAW_OFF + (Q8A ? SK_STAGES * SK_RAW : 0);
    const uint32_t bars = base + BAR_OFF;
    auto full_bar = [&](int s) { return bars + 8 * s; };
    auto empty_bar = [&](int s) { return bars + 8 * (SK_STAGES + s); };
    const uint32_t tfull = bars + 8 * (2 * SK_STAGES);
    auto raw_bar = [&](int s) { return bars + 8 * (2 * SK_STAGES + 1 + s); };  // Q8A: slot s landed
    uint32_t* tmem_slot =
        reinterpret_cast<uint32_t*>(smem + BAR_OFF + 8 * (2 * SK_STAGES + 1 + (Q8A ? SK_STAGES : 0)));
    float* part = reinterpret_cast<float*>(smem);  // split: [128][SK_PART_LD] partial tile (stages are free by then)

    if (threadIdx.x == 0) {
        prefetch_tmap(&maps.a);
        prefetch_tmap(&maps.b);
        if (Q8A) prefetch_tmap(&maps.as);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = blockIdx.x, split = blockIdx.y;
    const int nk = (p.K + SK_BK - 1) / SK_BK;
    const int kb0 = (int)((long)nk * split / p.splits), kb1 = (int)((long)nk * (split + 1) / p.splits);

    if (threadIdx.x == 0) {
        for (int s = 0; s < SK_STAGES; ++s) {
            mbar_init(full_bar(s), Q8A ? 2 : 1);  // Q8A: the B bytes' arrival and the converters'
            mbar_init(empty_bar(s), 1);
            if (Q8A) mbar_init(raw_bar(s), 1);
        }
        mbar_init(tfull, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(SK_BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    pdl_trigger();

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ TMA producer
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        int issued = 0;
        for (int kb = kb0; kb < kb1; ++kb, ++issued) {
            if (!mbar_wait(empty_bar(s), ph ^ 1, p.err, 21)) { ok = false; break; }
            const uint32_t sa = base + s * SK_STAGE, sb = sa + SK_A_BYTES;
            const int k0 = kb * SK_BK, m0 = mt * SK_BM;
            mbar_expect_tx(full_bar(s), Q8A ? SK_B_BYTES : SK_STAGE);
            if (Q8A) {  // quants and scales into the stage's raw slot, for the converters
                const uint32_t rq = base + RAW_OFF + s * SK_RAW, rsc = rq + SK_RAW_Q;
                mbar_expect_tx(raw_bar(s), SK_RAW_Q + 2 * SK_BM * 2);
                if (p.a_mn) {  // quants [K][M]: 128 (m) x 64 (k); scales [M / 32][K]: 64 (k) x 4
                    tma_load_2d(rq, &maps.a, m0, k0, raw_bar(s));
                    tma_load_2d(rsc, &maps.as, k0, m0 / 32, raw_bar(s));
                } else {       // quants [M][K]: 64 (k) x 128 (m); scales [K / 32][M]: 128 (m) x 2
                    tma_load_2d(rq, &maps.a, k0, m0, raw_bar(s));
                    tma_load_2d(rsc, &maps.as, m0, k0 / 32, raw_bar(s));
                }
            } else if (p.a_mn) {  // A stored [K][M]: two 64 (m) x 64 (k) boxes
                tma_load_2d(sa, &maps.a, m0, k0, full_bar(s));
                tma_load_2d(sa + 8192, &maps.a, m0 + 64, k0, full_bar(s));
            } else {       // A stored [M][K]: one 64 (k) x 128 (m) box
                tma_load_2d(sa, &maps.a, k0, m0, full_bar(s));
            }
            if (p.b_mn) tma_load_2d(sb, &maps.b, 0, k0, full_bar(s));  // [K][n]: 64 (n) x 64 (k)
            else tma_load_2d(sb, &maps.b, k0, 0, full_bar(s));         // [n][K]: 64 (k) x 64 (n)
            if (++s == SK_STAGES) { s = 0; ph ^= 1; }
        }
        if (!ok)  // drain what was issued before giving up
            for (int j = 0; j < SK_STAGES && issued - 1 - j >= 0; ++j) {
                const int i2 = issued - 1 - j;
                if (Q8A) mbar_wait_drain(raw_bar(i2 % SK_STAGES), (uint32_t)((i2 / SK_STAGES) & 1));
                mbar_wait(full_bar(i2 % SK_STAGES), (i2 / SK_STAGES) & 1, p.err, 25);
            }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ MMA issuer
        const uint32_t idesc = IDESC_F16_F32ACC | ((uint32_t)p.a_mn << 15) |
                               ((uint32_t)p.b_mn << 16) | ((uint32_t)(SK_BN >> 3) << 17) |
                               ((uint32_t)(SK_BM >> 4) << 24);
        const uint64_t a_desc0 = p.a_mn ? smem_desc(base, 8192, 1024) : smem_desc(base, 16, 1024);
        const uint64_t b_desc0 = p.b_mn ? smem_desc(base + SK_A_BYTES, 8192, 1024) : smem_desc(base + SK_A_BYTES, 16, 1024);
        const uint32_t a_step = (p.a_mn ? 2048 : 32) >> 4, b_step = (p.b_mn ? 2048 : 32) >> 4;
        int s = 0;
        uint32_t ph = 0;
        for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait(full_bar(s), ph, p.err, 22)) break;
            const uint64_t soff = (uint64_t)((s * SK_STAGE) >> 4);
#pragma unroll
            for (int k16 = 0; k16 < SK_BK / 16; ++k16)
                mma_f16(tmem, a_desc0 + soff + a_step * k16, b_desc0 + soff + b_step * k16, idesc,
                        (kb > kb0 || k16 > 0) ? 1u : 0u);
            mma_commit(empty_bar(s));
            if (++s == SK_STAGES) { s = 0; ph ^= 1; }
        }
        mma_commit(tfull);  // also covers an empty range: the epilogue then reads nothing
    } else if (Q8A && warp >= 6) {
        // ------------------------------------------------------------ Q8_0 converters
        // Slot s lands only after the MMA has released stage s (the producer waits for that
        // before reloading it), so the A tile may be overwritten then.  The four warps agree
        // (and have written the tile) before one thread counts them into the full barrier.
        const int ct = threadIdx.x - 6 * 32;
        int s = 0;
        uint32_t ph = 0;
        for (int kb = kb0; kb < kb1; ++kb) {
            bool got = mbar_wait(raw_bar(s), ph, p.err, 26);
            if (got) {
                if (p.a_mn) convert_q8_stage<SK_BM, true, 128>(smem, RAW_OFF + s * SK_RAW, s * SK_STAGE, ct);
                else convert_q8_stage<SK_BM, false, 128>(smem, RAW_OFF + s * SK_RAW, s * SK_STAGE, ct);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            }
            uint32_t all;
            asm volatile(
                "{\n\t.reg .pred p, q;\n\t"
                "setp.ne.u32 p, %1, 0;\n\t"
                "bar.red.and.pred q, 1, 128, p;\n\t"
                "selp.u32 %0, 1, 0, q;\n\t}"
                : "=r"(all)
                : "r"(got ? 1u : 0u)
                : "memory");
            if (!all) break;
            if (ct == 0) mbar_arrive(full_bar(s));
            if (++s == SK_STAGES) { s = 0; ph ^= 1; }
        }
    } else if (warp >= 2) {
        // ------------------------------------------------------------ epilogue
        const int quad = warp & 3;
        const int row = mt * SK_BM + quad * 32 + lane;
        bool ok = true;
        if (lane == 0) ok = mbar_wait(tfull, 0, p.err, 23);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const bool any = ok && kb1 > kb0;
        float v[SK_BN];
        for (int c = 0; c < SK_BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + c * 32, r);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[c * 32 + i] = any ? __uint_as_float(r[i]) * p.alpha : 0.f;
        }
        const bool in = row < p.M;
        if (p.splits == 1 && p.kind == SKINNY_ACC) {
            float* o = static_cast<float*>(p.out) + (long)row * p.ldo;
            if (in && any)
#pragma unroll
                for (int j = 0; j < SK_BN; ++j)
                    if (j < p.nb) o[j] += v[j];
        } else if (p.splits == 1 && p.kind == SKINNY_ACC_T) {
            float* o = static_cast<float*>(p.out) + row;
            if (in && any)
#pragma unroll
                for (int j = 0; j < SK_BN; ++j)
                    if (j < p.nb) o[(long)j * p.ldo] += v[j];  // lanes: consecutive rows
        } else if (p.splits == 1) {
            f16* o = static_cast<f16*>(p.out) + (long)row * p.ldo;
            if (in)
#pragma unroll
                for (int j = 0; j < SK_BN; j += 2)
                    if (j < p.nb) *reinterpret_cast<uint32_t*>(o + j) = pack_f16(v[j], v[j + 1]);
        } else {
            float* pr = part + (quad * 32 + lane) * SK_PART_LD;
#pragma unroll
            for (int j = 0; j < SK_BN; j += 4)
                if (j < p.nb) *reinterpret_cast<float4*>(pr + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (p.splits > 1) {
        // every thread of every CTA of the cluster passes both barriers (no early exit above)
        cluster_sync_all();
        const int S = p.splits, rank = (int)cluster_ctarank();
        const int rows_per = SK_BM / S, r0 = rank * rows_per, c4n = (p.nb + 3) / 4;
        const uint32_t part_s = smem_u32(part);
        // items run along the rows first for ACC_T (its rows are the gradient's columns)
        const bool trans = p.kind == SKINNY_ACC_T;
        for (int item = threadIdx.x; item < rows_per * c4n; item += NT) {
            const int rl = r0 + (trans ? item % rows_per : item / c4n), c4 = trans ? item / rows_per : item % c4n;
            const uint32_t off = part_s + (uint32_t)(rl * SK_PART_LD + 4 * c4) * 4;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int q = 0; q < S; ++q) {  // split order: the same sum whoever finished first
                const float4 t = ld_dsmem_f4(map_cta(off, (uint32_t)q));
                acc.x += t.x; acc.y += t.y; acc.z += t.z; acc.w += t.w;
            }
            const int grow = mt * SK_BM + rl;
            if (grow >= p.M) continue;
            const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
            if (p.kind == SKINNY_STORE) {
                *reinterpret_cast<uint2*>(static_cast<f16*>(p.out) + (long)grow * p.ldo + 4 * c4) =
                    make_uint2(pack_f16(acc.x, acc.y), pack_f16(acc.z, acc.w));
            } else if (p.kind == SKINNY_ACC) {
                float* o = static_cast<float*>(p.out) + (long)grow * p.ldo + 4 * c4;
                for (int j = 0; j < 4 && 4 * c4 + j < p.nb; ++j) o[j] += a4[j];
            } else {
                float* o = static_cast<float*>(p.out) + grow + (long)(4 * c4) * p.ldo;
                for (int j = 0; j < 4 && 4 * c4 + j < p.nb; ++j) o[(long)j * p.ldo] += a4[j];
            }
        }
        cluster_sync_all();  // peers keep their partials until every reader is done
    }
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(SK_BN));
}

int g_sms = 0;

}  // namespace

bool skinny_supported(const SkinnyArgs& a) {
    if (a.nb <= 0 || a.nb > SK_BN || a.M <= 0 || a.K <= 0) return false;
    if (a.kind == SKINNY_STORE && (a.nb & 3)) return false;
    if (a.Aq) {  // Q8_0 A: whole 32-blocks along K and along M (the scale boxes), 16-byte rows
        if (!a.Ad || a.K % 32 || a.M % 32 || a.lda % 16 || (a.ldad * 2) % 16 || (a.ldb * 2) % 16) return false;
        if ((reinterpret_cast<uintptr_t>(a.Aq) | reinterpret_cast<uintptr_t>(a.Ad) |
             reinterpret_cast<uintptr_t>(a.B)) & 15)
            return false;
        return a.kind != SKINNY_STORE || (!(a.ldo & 1) && !(reinterpret_cast<uintptr_t>(a.out) & 3));
    }
    if ((a.lda * 2) % 16 || (a.ldb * 2) % 16) return false;
    if ((reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.B)) & 15) return false;
    if (a.kind == SKINNY_STORE && ((a.ldo & 1) || (reinterpret_cast<uintptr_t>(a.out) & 3))) return false;
    return true;
}


void skinny_gemm(const SkinnyArgs& a, int* err, cudaStream_t s) {
    if (!skinny_supported(a)) throw std::runtime_error("skinny_gemm: unsupported operands");
    SkMaps maps;
    const bool q8 = a.Aq != nullptr;
    if (q8) {
        // quants: MN-major [K][M] (box 128 m x 64 k bytes), K-major [M][K] (box 64 k x 128 m);
        // scales one row per 32 quant columns: [M / 32][K] (box 64 k x 4) or [K / 32][M] (128 m x 2)
        if (a.a_mn) {
            tc_make_map_raw(&maps.a, a.Aq, false, a.K, a.M, a.lda, SK_BM, SK_BK);
            tc_make_map_raw(&maps.as, a.Ad, true, a.M / 32, a.K, a.ldad, SK_BK, SK_BM / 32);
        } else {
            tc_make_map_raw(&maps.a, a.Aq, false, a.M, a.K, a.lda, SK_BK, SK_BM);
            tc_make_map_raw(&maps.as, a.Ad, true, a.K / 32, a.M, a.ldad, SK_BM, 2);
        }
    } else {
        // A(m, k): MN-major stored [K][M] (box 64 m x 64 k), K-major stored [M][K] (box 64 k x 128 m)
        if (a.a_mn) tc_make_map(&maps.a, a.A, a.K, a.M, a.lda, 64, SK_BK);
        else tc_make_map(&maps.a, a.A, a.M, a.K, a.lda, SK_BK, SK_BM);
        maps.as = maps.a;
    }
    // B(k, n): MN-major stored [K][nb] (box 64 n x 64 k), K-major stored [nb][K] (box 64 k x 64 n)
    if (a.b_mn) tc_make_map(&maps.b, a.B, a.K, a.nb, a.ldb, SK_BN, SK_BK);
    else tc_make_map(&maps.b, a.B, a.nb, a.K, a.ldb, SK_BK, SK_BN);
    if (!g_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    }
    const int tiles = (a.M + SK_BM - 1) / SK_BM;
    const int nk = (a.K + SK_BK - 1) / SK_BK;
    // about two CTAs per SM (Q8_0 A: one, the converters take the other's registers)
    const int per_sm = q8 ? 1 : 2;
    int splits = a.splits > 0 ? a.splits : (per_sm * g_sms + tiles - 1) / tiles;
    if (splits > nk) splits = nk;
    if (splits < 1) splits = 1;
    {  // the split CTAs form one cluster: a power of two up to 8
        int c = 1;
        while (c * 2 <= splits && c * 2 <= 8) c *= 2;
        splits = c;
    }
    SkParams p;
    p.M = a.M; p.K = a.K; p.nb = a.nb; p.a_mn = a.a_mn ? 1 : 0; p.b_mn = a.b_mn ? 1 : 0;
    p.kind = a.kind; p.alpha = a.alpha; p.out = a.out; p.ldo = a.ldo;
    p.splits = splits; p.err = err;
    static DeviceOnce once;
    once([] {
        cudaFuncSetAttribute(skinny_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM);
        cudaFuncSetAttribute(skinny_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM_Q8);
    });
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles, splits, 1);
    cfg.blockDim = dim3(q8 ? SK_THREADS_Q8 : SK_THREADS, 1, 1);
    cfg.dynamicSmemBytes = q8 ? SK_SMEM_Q8 : SK_SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = splits;
    attr[0].val.clusterDim.z = 1;
    pdl_attr(attr[1]);
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaLaunchKernelEx(&cfg, q8 ? skinny_kernel<true> : skinny_kernel<false>, maps, p);
}

}  // namespace act
