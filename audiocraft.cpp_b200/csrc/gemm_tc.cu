// gemm_tc.cu -- dense projection GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// C[m][n] = epilogue( sum_k A[m][k] B(n,k) ) with A K-major (activations / output gradients,
// row-major [M][K]) and B either K-major (frozen weight [N][K]: forward Y = X W^T) or MN-major
// (frozen weight read as [K][N]: input gradient dX = dY W).  A second K segment (A2, B2)
// carries the LoRA rank block, so  Y = [X | sXA^T] [W | B]^T  and  dX = [dY | dU] [W ; A]
// are each one pass over the tile.
//
// Persistent, warp-specialised CTA (one per SM):
//   warp 0      TMA producer (one elected thread): A box 128x64, B box 256x64 (or 4 boxes of
//               64x64 for MN-major B), 128-byte swizzle, into a 4-stage ring
//   warp 1      MMA issuer (one thread): tcgen05.mma.cta_group::1.kind::f16, 128 x BN x 16,
//               fp32 accumulators in TMEM, two accumulator buffers so the epilogue of tile i
//               overlaps the mainloop of tile i+1
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, fused epilogue, 16-byte stores
// Every mbarrier wait is bounded (globaltimer); on expiry the CTA records an error code,
// drains what it issued and returns, so a logic error cannot hang the device.
// No cluster launch: every CTA issues its own TMA loads for its own tiles.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace act {

namespace {

using namespace tc;

constexpr int BM = 128;
constexpr int BKE = 64;  // K elements per stage (one 128-byte swizzle row)
constexpr int EPI_WARPS = 4;
constexpr int NTHREADS = (2 + EPI_WARPS) * 32;
// The 2-CTA kernel drains each accumulator with two warps per TMEM lane quarter (one per half
// of the tile's columns): the epilogue of a tile is latency-bound per warp, so twice the warps
// finish it in about half the time.
constexpr int EPI_WARPS2 = 8;
constexpr int NTHREADS2 = (2 + EPI_WARPS2) * 32;

struct TcParams {
    int M, N, K1, K2;
    int num_m, num_n;
    int mode;
    float alpha;
    const float* colscale;
    void* out;
    long ldo;
    const float* resid;
    long ldr;
    f16* aux;
    f16* out_h;
    long ldaux;
    const f16* auxin;
    long ldauxin;
    const float* colscale2;
    const float* bias;
    const float* rope;
    int rope_T, rope_cols;
    int nvalid, mvalid;
    int* err;
    // 2-CTA kernel, stream-K instantiation: fp32 partial pair tiles [pair][rank][warp][4096] and
    // one ready counter per [pair][rank]
    float* sk_part;
    int* sk_flag;
    // 2-CTA kernel, Q8_0 instantiation: bit i set when K segment i + 1 reads Q8_0 weights
    int q8mask;
    // 2-CTA kernel: A2 is the previous kernel's output; only the producer waits for that kernel,
    // right before its first A2 load (everything else the CTA reads is older)
    int late_wait;
};

struct TcMaps {
    CUtensorMap a1, b1, a2, b2;
    CUtensorMap s1, s2;   // Q8_0 segments: block scales (b1 / b2 then map the quants)
    CUtensorMap out, aux;  // epilogue stores: box 32 x 32, swizzle 128 B (fp32) / 64 B (f16)
    CUtensorMap out_h;    // f16 copy of an fp32 output
};

// Epilogue staging, per epilogue warp: a 32-row x 128-byte tile for the output chunk (32 fp32
// or 32 f16 columns; 128-byte swizzle) and a 32 x 64-byte tile for f16 side outputs/inputs
// (64-byte swizzle).  Both leave shared memory through TMA bulk tensor stores.
constexpr int EPI_OUT_BYTES = 32 * 128;
constexpr int EPI_AUX_BYTES = 32 * 64;
constexpr int EPI_SMEM = EPI_WARPS * (EPI_OUT_BYTES + EPI_AUX_BYTES);

template <int BN>
struct TcCfg {
    static constexpr int A_BYTES = BM * BKE * 2;
    static constexpr int B_BYTES = BN * BKE * 2;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int STAGES = BN == 256 ? 4 : 6;
    static constexpr int SMEM = STAGES * STAGE + EPI_SMEM + 1024 /*align*/ + 256 /*barriers*/;
    static constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulator buffers
};

// ---------------------------------------------------------------------------------------
// Epilogue.  After tcgen05.ld each lane holds 32 consecutive columns of ONE row.  The warp
// writes the chunk into its swizzled staging tile (conflict-free: the 16-byte unit u of row r
// sits at unit u ^ f(r)) and one lane issues a TMA bulk tensor store, which clips rows past the
// tensor's extent.  Residual / accumulator / GELU inputs come in through the same tiles with
// coalesced loads (one 128-byte row segment per 8 or 4 lanes).

// byte offset of 16-byte unit u of row r: 128-byte swizzle (rows of 128 B, tile 1024-aligned)
__device__ __forceinline__ uint32_t sw128(int r, int u) { return r * 128 + ((u ^ (r & 7)) << 4); }
// 64-byte swizzle (rows of 64 B, tile 512-aligned)
__device__ __forceinline__ uint32_t sw64(int r, int u) { return r * 64 + ((u ^ ((r >> 1) & 3)) << 4); }

struct EpiTiles {
    unsigned char* o;  // output chunk tile (EPI_OUT_BYTES)
    unsigned char* x;  // f16 side tile (EPI_AUX_BYTES)
    uint32_t o_s, x_s; // their shared-state-space addresses
};

// previous bulk stores of this warp (all issued by lane 0) have finished reading the tiles
__device__ __forceinline__ void tiles_free(int lane) {
    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    __syncwarp();
}

__device__ __forceinline__ void tile_store(const CUtensorMap* map, uint32_t src, int x, int y, int lane) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) {
        asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                     ::"l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(src)
                     : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
}

__device__ __forceinline__ void put_row_f32(unsigned char* t, int lane, const float* v) {
#pragma unroll
    for (int u = 0; u < 8; ++u)
        *reinterpret_cast<float4*>(t + sw128(lane, u)) = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
}

__device__ __forceinline__ void add_row_f32(const unsigned char* t, int lane, float* v) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const float4 r = *reinterpret_cast<const float4*>(t + sw128(lane, u));
        v[4 * u] += r.x; v[4 * u + 1] += r.y; v[4 * u + 2] += r.z; v[4 * u + 3] += r.w;
    }
}

// 32 f16 of this lane's row into a 64-byte-swizzled tile
__device__ __forceinline__ void put_row_b16(unsigned char* t, int lane, const float* v) {
#pragma unroll
    for (int u = 0; u < 4; ++u)
        *reinterpret_cast<uint4*>(t + sw64(lane, u)) =
            make_uint4(pack_f16(v[8 * u], v[8 * u + 1]), pack_f16(v[8 * u + 2], v[8 * u + 3]),
                       pack_f16(v[8 * u + 4], v[8 * u + 5]), pack_f16(v[8 * u + 6], v[8 * u + 7]));
}

__device__ __forceinline__ void get_row_b16(const unsigned char* t, int lane, float* v) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const uint4 q = *reinterpret_cast<const uint4*>(t + sw64(lane, u));
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 x = unpack_f16(w[j]);
            v[8 * u + 2 * j] = x.x;
            v[8 * u + 2 * j + 1] = x.y;
        }
    }
}

// Epilogue inputs read per chunk: fp32 residual / accumulator rows (RESID, ACCUM) or f16 GELU
// pre-activations (GELU_BWD).  They are fetched one chunk ahead into registers as coalesced
// 128-byte row segments, so their latency overlaps the previous chunk, then staged in the tile.
// Kind 3: the RoPE (cos, sin) pairs of a f16-store chunk with rotary columns, loaded per lane
// (its own row) from the position table, which does not stay in L1 beside the operand stages.
__device__ __forceinline__ int epi_input_kind(const TcParams& p) {
    return (p.mode == EPI_RESID_F32 || p.mode == EPI_ACCUM_F32) ? 1
           : (p.mode == EPI_GELU_BWD || p.mode == EPI_GELU_BWD_D) ? 2
           : p.rope ? 3 : 0;
}

// chunk rows m_base .. m_base+rows-1 (rows <= 0: nothing), columns n .. n+31
__device__ __forceinline__ void fetch_input(const TcParams& p, int kind, int m_base, int rows, int n, int lane,
                                            float4* pre) {
    if (kind == 1) {
        const bool acc = p.mode == EPI_ACCUM_F32;
        const float* g = acc ? static_cast<const float*>(p.out) : p.resid;
        const long ld = acc ? p.ldo : p.ldr;
#pragma unroll
        for (int it = 0; it < 8; ++it) {
            const int r = it * 4 + (lane >> 3), u = lane & 7;
            pre[it] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r < rows) pre[it] = *reinterpret_cast<const float4*>(g + (long)(m_base + r) * ld + n + 4 * u);
        }
    } else if (kind == 2) {
#pragma unroll
        for (int it = 0; it < 4; ++it) {
            const int r = it * 8 + (lane >> 2), u = lane & 3;
            pre[it] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r < rows)
                pre[it] = *reinterpret_cast<const float4*>(p.auxin + (long)(m_base + r) * p.ldauxin + n + 8 * u);
        }
    } else if (kind == 3) {
        // 16 (cos, sin) pairs of this lane's position for the chunk's columns within its head
        if (rows > 0 && n < p.rope_cols) {
            const float4* tt = reinterpret_cast<const float4*>(p.rope + (long)((m_base + lane) % p.rope_T) * 64 + n % 64);
#pragma unroll
            for (int it = 0; it < 8; ++it) pre[it] = tt[it];
        }
    }
}

__device__ __forceinline__ void stage_input(int kind, const float4* pre, const EpiTiles& t, int lane) {
    if (kind == 1) {
#pragma unroll
        for (int it = 0; it < 8; ++it)
            *reinterpret_cast<float4*>(t.o + sw128(it * 4 + (lane >> 3), lane & 7)) = pre[it];
    } else if (kind == 2) {
#pragma unroll
        for (int it = 0; it < 4; ++it)
            *reinterpret_cast<float4*>(t.x + sw64(it * 8 + (lane >> 2), lane & 3)) = pre[it];
    } else if (kind == 3) {  // the lane's own row of the output tile, read back by the same lane
#pragma unroll
        for (int it = 0; it < 8; ++it) *reinterpret_cast<float4*>(t.o + sw128(lane, it)) = pre[it];
    }
}

// Warp-collective epilogue of the 32 x 32 chunk rows m_base .. m_base+31 (the first `rows`
// valid), columns n .. n+31; lane l holds row m_base + l in v[].  The caller has made the
// tiles `t` free.
__device__ __forceinline__ void epilogue_warp32(const TcParams& p, const TcMaps& maps, int m_base, int rows, int n,
                                                float* v, const EpiTiles& t, int lane) {
    if (p.alpha != 1.0f)
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= p.alpha;
    if (p.colscale) {
        const float4* cs = reinterpret_cast<const float4*>(p.colscale + n);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 c = cs[i];
            v[4 * i] *= c.x; v[4 * i + 1] *= c.y; v[4 * i + 2] *= c.z; v[4 * i + 3] *= c.w;
        }
    }
    if (p.aux && p.mode != EPI_GELU && p.mode != EPI_GELU_D) {
        put_row_b16(t.x, lane, v);
        tile_store(&maps.aux, t.x_s, n, m_base, lane);
    }
    if (p.rope && n < p.rope_cols) {  // 32 columns inside one 64-wide head: 16 rotary pairs
        // (cos, sin) pairs staged in this lane's row of the output tile (input kind 3)
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const float4 c = *reinterpret_cast<const float4*>(t.o + sw128(lane, u));
            const float x0 = v[4 * u], x1 = v[4 * u + 1], x2 = v[4 * u + 2], x3 = v[4 * u + 3];
            v[4 * u] = x0 * c.x - x1 * c.y;
            v[4 * u + 1] = x0 * c.y + x1 * c.x;
            v[4 * u + 2] = x2 * c.z - x3 * c.w;
            v[4 * u + 3] = x2 * c.w + x3 * c.z;
        }
        __syncwarp();  // every lane has its pairs before the output overwrites the tile
    }
    if (p.mode == EPI_STORE_F32 || p.mode == EPI_ACCUM_F32 || p.mode == EPI_RESID_F32) {
        if (p.mode != EPI_STORE_F32) add_row_f32(t.o, lane, v);  // residual / accumulator already staged in the tile
        put_row_f32(t.o, lane, v);
        tile_store(&maps.out, t.o_s, n, m_base, lane);
        if (p.out_h) {
            if (p.aux) tiles_free(lane);  // the side tile is still being read by this chunk's aux store
            put_row_b16(t.x, lane, v);
            tile_store(&maps.out_h, t.x_s, n, m_base, lane);
        }
        return;
    }
    if (p.mode == EPI_BIAS_F16) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += p.bias[n + i];
    } else if (p.mode == EPI_GELU) {
        // the stored pre-activation is f16; the activation and its backward use that value
        put_row_b16(t.x, lane, v);
        get_row_b16(t.x, lane, v);
        tile_store(&maps.aux, t.x_s, n, m_base, lane);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = gelu_as(v[i]);
    } else if (p.mode == EPI_GELU_D) {
        // gelu' of the f16-rounded pre-activation goes to aux, gelu of it to the output
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            float d8[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float g;
                gelu_as_pair(__half2float(__float2half_rn(v[8 * u + j])), g, d8[j]);
                v[8 * u + j] = g;
            }
            *reinterpret_cast<uint4*>(t.x + sw64(lane, u)) =
                make_uint4(pack_f16(d8[0], d8[1]), pack_f16(d8[2], d8[3]), pack_f16(d8[4], d8[5]),
                           pack_f16(d8[6], d8[7]));
        }
        tile_store(&maps.aux, t.x_s, n, m_base, lane);
    } else if (p.mode == EPI_GELU_BWD || p.mode == EPI_GELU_BWD_D) {
        float z[32];
        get_row_b16(t.x, lane, z);  // pre-activation (or its gelu') already staged in the side tile
        if (p.mode == EPI_GELU_BWD) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= gelu_as_grad(z[i]);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= z[i];
        }
        if (p.colscale2)
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= p.colscale2[n + i];
    }
    put_row_b16(t.o, lane, v);
    tile_store(&maps.out, t.o_s, n, m_base, lane);
}

// All chunks of one accumulator tile (NCH x 32 columns from TMEM row address `trow`).  The
// next chunk's inputs (this tile's, or chunk 0 of the warp's next tile) are fetched while the
// current one is finished.
// `part` (shared memory, may be null): an fp32 partial of the same accumulator fragment, added
// before the epilogue; chunk c, float4 g of lane l at part[(c * 8 + g) * 32 + l].
template <int NCH>
__device__ __forceinline__ void epilogue_tile(const TcParams& p, const TcMaps& maps, uint32_t trow, int m_base,
                                              int rows, int n0, int next_m_base, int next_rows, int next_n0,
                                              const EpiTiles& t, int lane, float4* pre,
                                              const float4* part = nullptr) {
    const int kind = epi_input_kind(p);
    for (int c = 0; c < NCH; ++c) {
        uint32_t r[32];
        tmem_ld32(trow + c * 32, r);
        if (part) {
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                const float4 q = part[(c * 8 + g) * 32 + lane];
                r[4 * g] = __float_as_uint(__uint_as_float(r[4 * g]) + q.x);
                r[4 * g + 1] = __float_as_uint(__uint_as_float(r[4 * g + 1]) + q.y);
                r[4 * g + 2] = __float_as_uint(__uint_as_float(r[4 * g + 2]) + q.z);
                r[4 * g + 3] = __float_as_uint(__uint_as_float(r[4 * g + 3]) + q.w);
            }
        }
        const int n = n0 + c * 32;
        if (rows > 0) tiles_free(lane);
        if (kind) {
            if (rows > 0) stage_input(kind, pre, t, lane);
            if (c + 1 < NCH) fetch_input(p, kind, m_base, rows, n + 32, lane, pre);
            else fetch_input(p, kind, next_m_base, next_rows, next_n0, lane, pre);
            __syncwarp();
        }
        if (rows > 0) epilogue_warp32(p, maps, m_base, rows, n, reinterpret_cast<float*>(r), t, lane);
    }
}

template <int BN, bool B_MN>
__global__ void __launch_bounds__(NTHREADS, 1) gemm_tc_kernel(const __grid_constant__ TcMaps maps, const TcParams p) {
    using Cfg = TcCfg<BN>;
    constexpr int S = Cfg::STAGES;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023) & ~1023u;
    unsigned char* smem = smem_raw + (base - raw);
    const uint32_t bars = base + S * Cfg::STAGE + EPI_SMEM;
    // barrier layout: full[S], empty[S], tfull[2], tempty[2], drain, then the TMEM address
    auto full_bar = [&](int s) { return bars + 8 * s; };
    auto empty_bar = [&](int s) { return bars + 8 * (S + s); };
    auto tfull_bar = [&](int a) { return bars + 8 * (2 * S + a); };
    auto tempty_bar = [&](int a) { return bars + 8 * (2 * S + 2 + a); };
    const uint32_t drain_bar = bars + 8 * (2 * S + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S * Cfg::STAGE + EPI_SMEM + 8 * (2 * S + 5));

    if (threadIdx.x == 0) {
        prefetch_tmap(&maps.a1);
        prefetch_tmap(&maps.b1);
        prefetch_tmap(&maps.a2);
        prefetch_tmap(&maps.b2);
        prefetch_tmap(&maps.out);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), EPI_WARPS);
        }
        mbar_init(drain_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(Cfg::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();
    pdl_trigger();

    const int nk1 = (p.K1 + BKE - 1) / BKE, nk2 = (p.K2 + BKE - 1) / BKE, nk = nk1 + nk2;
    const int ntiles = p.num_m * p.num_n;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ TMA producer
        int it = 0, s = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            const int mb = tile % p.num_m, nb = tile / p.num_m;
            for (int kb = 0; kb < nk; ++kb, ++it) {
                if (!mbar_wait(empty_bar(s), ph ^ 1, p.err, 1)) { ok = false; break; }
                const bool seg2 = kb >= nk1;
                const CUtensorMap* ma = seg2 ? &maps.a2 : &maps.a1;
                const CUtensorMap* mbm = seg2 ? &maps.b2 : &maps.b1;
                const int k0 = (seg2 ? kb - nk1 : kb) * BKE;
                const uint32_t sa = base + s * Cfg::STAGE, sb = sa + Cfg::A_BYTES;
                mbar_expect_tx(full_bar(s), Cfg::STAGE);
                tma_load_2d(sa, ma, k0, mb * BM, full_bar(s));
                if (B_MN) {
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * 8192, mbm, nb * BN + 64 * j, k0, full_bar(s));
                } else {
                    tma_load_2d(sb, mbm, k0, nb * BN, full_bar(s));
                }
                if (++s == S) { s = 0; ph ^= 1; }
            }
        }
        // drain: wait until every stage this thread filled has landed
        if (!ok)
            for (int j = 0; j < S && it - 1 - j >= 0; ++j) {
                const int i2 = it - 1 - j;
                mbar_wait(full_bar(i2 % S), (i2 / S) & 1, p.err, 5);
            }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ MMA issuer
        const uint32_t idesc = IDESC_F16_F32ACC | ((B_MN ? 1u : 0u) << 16) |
                               ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
        // Stage-0 descriptors; a stage offset or a k16 step is added to the 14-bit start-address
        // field (shared-memory addresses stay below 256 KB, so the field cannot carry over).
        const uint64_t a_desc0 = smem_desc(base, 16, 1024);
        const uint64_t b_desc0 = B_MN ? smem_desc(base + Cfg::A_BYTES, 8192, 1024)
                                      : smem_desc(base + Cfg::A_BYTES, 16, 1024);
        constexpr uint32_t A_STEP = 32 >> 4, B_STEP = (B_MN ? 2048 : 32) >> 4;
        int s = 0, u = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++u) {
            const int a = u & 1;
            ok = mbar_wait(tempty_bar(a), ((u >> 1) & 1) ^ 1, p.err, 2);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t tacc = tmem_base + a * BN;
            for (int kb = 0; kb < nk; ++kb) {
                if (!mbar_wait(full_bar(s), ph, p.err, 3)) { ok = false; break; }
                const uint64_t soff = (uint64_t)((s * Cfg::STAGE) >> 4);
                const uint64_t ad = a_desc0 + soff, bd = b_desc0 + soff;
                const int kv = kb >= nk1 ? p.K2 - (kb - nk1) * BKE : BKE;
                if (kv >= BKE) {
#pragma unroll
                    for (int k16 = 0; k16 < BKE / 16; ++k16)
                        mma_f16(tacc, ad + A_STEP * k16, bd + B_STEP * k16, idesc, (kb | k16) ? 1u : 0u);
                } else {
                    for (int k16 = 0; k16 < (kv + 15) / 16; ++k16)
                        mma_f16(tacc, ad + A_STEP * k16, bd + B_STEP * k16, idesc, (kb | k16) ? 1u : 0u);
                }
                mma_commit(empty_bar(s));
                if (++s == S) { s = 0; ph ^= 1; }
            }
            if (!ok) break;
            mma_commit(tfull_bar(a));
        }
        // drain: all issued MMAs complete before TMEM is released
        mma_commit(drain_bar);
        mbar_wait(drain_bar, 0, p.err, 6);
    } else if (warp >= 2) {
        // ------------------------------------------------------------ epilogue
        const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31
        EpiTiles tiles;
        tiles.o = smem + S * Cfg::STAGE + (warp - 2) * EPI_OUT_BYTES;
        tiles.x = smem + S * Cfg::STAGE + EPI_WARPS * EPI_OUT_BYTES + (warp - 2) * EPI_AUX_BYTES;
        tiles.o_s = smem_u32(tiles.o);
        tiles.x_s = smem_u32(tiles.x);
        const int mlim = min(p.M, p.mvalid);
        auto tile_rows = [&](int tl, int& m_base, int& rows, int& n0) {
            m_base = (tl % p.num_m) * BM + quad * 32;
            rows = tl < ntiles ? max(0, min(32, mlim - m_base)) : 0;
            n0 = (tl / p.num_m) * BN;
        };
        float4 pre[8];
        {
            int mb0, r0, n00;
            tile_rows(blockIdx.x, mb0, r0, n00);
            fetch_input(p, epi_input_kind(p), mb0, r0, n00, lane, pre);
        }
        int u = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++u) {
            const int a = u & 1;
            bool ok = true;
            if (lane == 0) ok = mbar_wait(tfull_bar(a), (u >> 1) & 1, p.err, 4);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            int m_base, rows, n0, nm, nr, nn;
            tile_rows(tile, m_base, rows, n0);
            tile_rows(tile + gridDim.x, nm, nr, nn);
            epilogue_tile<BN / 32>(p, maps, tmem_base + ((uint32_t)(quad * 32) << 16) + a * BN, m_base, rows, n0, nm,
                                   nr, nn, tiles, lane, pre);
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(a));
        }
        // the staging tiles have been read; the stores themselves complete with the grid
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    __syncwarp();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(Cfg::TMEM_COLS));
}

// ---------------------------------------------------------------------------------------
// 2-CTA variant: a cluster of two CTAs computes a 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256).  Each CTA stages its own 128 rows of A and its
// own 128 rows of B (half of the tile's columns); the leader CTA (cluster rank 0) issues the
// MMAs, which read both CTAs' shared memory and write both CTAs' TMEM (rows 0..127 in the
// leader, 128..255 in the peer).  Twice the FLOPs per byte staged from L2 of the 1-CTA
// 128 x 256 tile, which is what bounds that kernel.  Loads are plain per-CTA TMA loads whose
// completion bytes are posted to the leader's barrier; the leader signals the peer's barriers
// with ordinary commits addressed through mapa.
// Each CTA drains its 128 accumulator rows with 8 epilogue warps (warps 2..9): two per TMEM
// lane quarter, each taking half of the tile's columns.

// BNP: output columns of a pair tile (256 or 128); each CTA stages BNP / 2 rows of B.
// Q8: B arrives as Q8_0 weights.  The quants (biased to unsigned, BH x 64 bytes per k-block) and
// their f16 block scales (BH x 2 values) come by TMA into a ring of raw slots of their own, which
// the converter warps keep filled RSLOTS k-blocks ahead (the weights do not wait for the MMA to
// free a stage); once a stage is free the CW converter warps turn its raw slot into the f16
// operand tile.  The conversion is redone for every row tile, about two instructions per weight
// element, so it gets as many warps as the epilogue: the Q8_0 kernel drains TMEM with 4
// epilogue warps (one per lane quarter, all columns) and converts with 4, in the same 320
// threads, and keeps one operand stage fewer to make room for the raw ring.
template <int BNP, bool Q8 = false>
struct Tc2Cfg {
    static constexpr int BH = BNP / 2;
    static constexpr int EW = Q8 ? 4 : EPI_WARPS2;  // epilogue warps
    static constexpr int CW = Q8 ? 4 : 0;           // converter warps
    static constexpr int A_BYTES = BM * BKE * 2;
    static constexpr int B_BYTES = BH * BKE * 2;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int STAGES = (BNP == 256 ? 5 : 7) - (Q8 ? 1 : 0);
    static constexpr int EPI = EW * (EPI_OUT_BYTES + EPI_AUX_BYTES);
    static constexpr int Q_BYTES = BH * BKE;         // quants of this CTA's half of B, one k-block
    static constexpr int S_BYTES = 2 * BH * 2;       // their f16 scales (BH * 64 / 32)
    static constexpr int RAW = Q8 ? (Q_BYTES + S_BYTES + 1023) / 1024 * 1024 : 0;
    static constexpr int RSLOTS = Q8 ? 8 : 0;
    static constexpr int SMEM = STAGES * STAGE + EPI + RSLOTS * RAW + 1024 + 256;
    static constexpr int THREADS = (2 + EW + CW) * 32;
    static constexpr uint32_t TMEM_COLS = 2 * BNP;
};

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of the same shared-memory offset in cluster CTA `rank`
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                                 uint32_t leader_bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(leader_bar)
        : "memory");
}

__device__ __forceinline__ void mma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit_pair(uint32_t cluster_bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
                 : "memory");
}

// Work of one CTA pair.  Whole tiles (sk = 0): tiles pair, pair + npairs, ...  Stream-K
// (sk = 1): the pair takes units [pair * U / npairs, (pair + 1) * U / npairs) of the U = tiles x
// k-blocks units, tile-major.  The host enables stream-K only when there are at least as many
// tiles as pairs, so every range covers >= nk units: a tile is split at most once, between the
// end of pair p's range (its first k-blocks, the pair's LAST item: SK_PART_IN) and the start
// of pair p+1's (its last k-blocks, that pair's FIRST item: SK_PART_OUT).  Pair p+1 finishes
// its part early and leaves the fp32 partial in slot p+1; pair p adds it in its epilogue.
enum { SK_FULL = 0, SK_PART_OUT = 1, SK_PART_IN = 2 };

struct PairWork {
    int nk, ntiles, npairs, tile;
    long u, end;
    bool sk;
    __device__ PairWork(int sk_, int nk_, int ntiles_, int pair, int npairs_)
        : nk(nk_), ntiles(ntiles_), npairs(npairs_), tile(pair), u(0), end(0), sk(sk_ != 0) {
        if (sk) {
            const long units = (long)ntiles * nk;
            u = units * pair / npairs;
            end = units * (pair + 1) / npairs;
        }
    }
    // next item: tile, k-block range [kb0, kb1), role; false when the pair is done
    __device__ bool next(int& t, int& kb0, int& kb1, int& role) {
        if (!sk) {
            if (tile >= ntiles) return false;
            t = tile; kb0 = 0; kb1 = nk; role = SK_FULL;
            tile += npairs;
            return true;
        }
        if (u >= end) return false;
        t = (int)(u / nk);
        kb0 = (int)(u - (long)t * nk);
        kb1 = (int)min((long)nk, kb0 + (end - u));
        role = kb0 > 0 ? SK_PART_OUT : (kb1 < nk ? SK_PART_IN : SK_FULL);
        u += kb1 - kb0;
        return true;
    }
};

// stream-K partial of one epilogue warp: 32 rows x 128 columns, fp32, TMEM-fragment order
// A stream-K partial is one CTA's 128 x 256 fp32 accumulator (128 KB: 4 stages of the 256-wide
// ring), stored epilogue-warp-major: each warp's 32 rows x its columns, chunk by chunk.
constexpr int SK_CTA_FLOATS = 128 * 256;
constexpr int SK_CTA_BYTES = SK_CTA_FLOATS * 4;

template <int BN2, bool B_MN, bool SK, bool Q8>
__global__ void __launch_bounds__(Tc2Cfg<BN2, Q8>::THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ TcMaps maps, const TcParams p) {
    using Cfg = Tc2Cfg<BN2, Q8>;
    constexpr int BH2 = Cfg::BH;
    constexpr int S = Cfg::STAGES;
    constexpr int R = Cfg::RSLOTS;
    static_assert(!SK || S * Cfg::STAGE >= SK_CTA_BYTES, "a stream-K partial must fit in the operand ring");
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023) & ~1023u;
    unsigned char* smem = smem_raw + (base - raw);
    const uint32_t raw_off = S * Cfg::STAGE + Cfg::EPI;  // Q8: the raw ring
    const uint32_t bars = base + raw_off + R * Cfg::RAW;
    auto full_bar = [&](int s) { return bars + 8 * s; };
    auto empty_bar = [&](int s) { return bars + 8 * (S + s); };
    auto tfull_bar = [&](int a) { return bars + 8 * (2 * S + a); };
    auto tempty_bar = [&](int a) { return bars + 8 * (2 * S + 2 + a); };
    const uint32_t drain_bar = bars + 8 * (2 * S + 4);
    const uint32_t part_bar = bars + 8 * (2 * S + 5);  // stream-K partial landed in the stages
    auto raw_bar = [&](int r) { return bars + 8 * (2 * S + 6 + r); };  // Q8: raw slot r landed (this CTA)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + raw_off + R * Cfg::RAW + 8 * (2 * S + 6 + R));
    // Q8: 16 bytes that the peer CTA's converters copy to the leader to count into full_bar
    constexpr uint32_t SIG_OFF = (8 * (2 * S + 6 + R) + 4 + 15) / 16 * 16;

    if (threadIdx.x == 0) {
        prefetch_tmap(&maps.a1);
        prefetch_tmap(&maps.b1);
        prefetch_tmap(&maps.a2);
        prefetch_tmap(&maps.b2);
        prefetch_tmap(&maps.out);
        if (Q8) {
            prefetch_tmap(&maps.s1);
            prefetch_tmap(&maps.s2);
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            // leader: one arrive_expect_tx for both CTAs' bytes (Q8: plus the leader's converters'
            // arrival; the peer's converters count in through the 16 bytes they copy here)
            mbar_init(full_bar(s), Q8 ? 2 : 1);
            mbar_init(empty_bar(s), 1);  // each CTA: one commit from the leader
        }
        for (int r = 0; r < R; ++r) mbar_init(raw_bar(r), 1);
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), 2 * Cfg::EW);  // leader: both CTAs' epilogue warps
        }
        mbar_init(drain_bar, 1);
        mbar_init(part_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(Cfg::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem_base = *tmem_slot;
    // late_wait: the previous kernel writes only A2, and it started after everything older had
    // completed (every kernel here waits before it triggers), so the CTA may stream A1 / B1 and
    // read its epilogue inputs now; the producer waits for the previous kernel before its first
    // A2 load, and every global write of the CTA follows that load through the MMA pipeline
    if (!p.late_wait) pdl_wait();
    pdl_trigger();

    const int nk1 = (p.K1 + BKE - 1) / BKE, nk2 = (p.K2 + BKE - 1) / BKE, nk = nk1 + nk2;
    const int num_m2 = (p.M + 2 * BM - 1) / (2 * BM);
    const int ntiles = num_m2 * p.num_n;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ TMA producer (both CTAs)
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        PairWork w(SK ? 1 : 0, nk, ntiles, pair, npairs);
        int tile, kb0, kb1, role = SK_FULL;
        // Q8: the raw ring.  Conv k-block i (the i-th Q8_0 k-block of the schedule) uses slot
        // i % R.  Waiting for stage s's release proves that the k-block S stages back has been
        // converted, so its slot is free: with each Q8_0 k-block this thread issues the quants of
        // the one R - S conv k-blocks ahead (the first R - S before the loop).
        PairWork ahead(SK ? 1 : 0, nk, ntiles, pair, npairs);
        int a_tile = 0, a_kb = 0, a_kb1 = 0, a_role, raw_issued = 0;
        auto issue_raw = [&]() {
            for (;;) {
                while (a_kb >= a_kb1)
                    if (!ahead.next(a_tile, a_kb, a_kb1, a_role)) return;
                const int k = a_kb++;
                if (!((p.q8mask >> (k >= nk1 ? 1 : 0)) & 1)) continue;
                const bool seg2 = k >= nk1;
                const int k0 = (seg2 ? k - nk1 : k) * BKE;
                const int n0 = (a_tile / num_m2) * BN2 + (int)rank * BH2;
                const CUtensorMap* mq = seg2 ? &maps.b2 : &maps.b1;
                const CUtensorMap* msc = seg2 ? &maps.s2 : &maps.s1;
                const int slot = raw_issued++ % R;
                const uint32_t rq = base + raw_off + slot * Cfg::RAW, rsc = rq + Cfg::Q_BYTES;
                mbar_expect_tx(raw_bar(slot), Cfg::Q_BYTES + Cfg::S_BYTES);
                if (B_MN) {
                    tma_load_2d(rq, mq, n0, k0, raw_bar(slot));
                    tma_load_2d(rsc, msc, k0, n0 / 32, raw_bar(slot));
                } else {
                    tma_load_2d(rq, mq, k0, n0, raw_bar(slot));
                    tma_load_2d(rsc, msc, n0, k0 / 32, raw_bar(slot));
                }
                return;
            }
        };
        if (Q8)
            for (int i = 0; i < R - S; ++i) issue_raw();
        bool waited = !p.late_wait;
        while (ok && w.next(tile, kb0, kb1, role)) {
            const int mb = tile % num_m2, nb = tile / num_m2;
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(empty_bar(s), ph ^ 1, p.err, 11)) { ok = false; break; }
                const bool seg2 = kb >= nk1;
                if (seg2 && !waited) {
                    pdl_wait();  // A2 is the previous kernel's output
                    waited = true;
                }
                const CUtensorMap* ma = seg2 ? &maps.a2 : &maps.a1;
                const CUtensorMap* mbm = seg2 ? &maps.b2 : &maps.b1;
                const int k0 = (seg2 ? kb - nk1 : kb) * BKE;
                const uint32_t sa = base + s * Cfg::STAGE, sb = sa + Cfg::A_BYTES;
                const uint32_t lbar = map_rank(full_bar(s), 0);
                const int n0 = nb * BN2 + rank * BH2;
                if (Q8 && ((p.q8mask >> (seg2 ? 1 : 0)) & 1)) {
                    // A only: B's quants come through the raw ring, for the converters
                    if (rank == 0) mbar_expect_tx(full_bar(s), 2 * Cfg::A_BYTES + 16);
                    tma_load_2d_pair(sa, ma, k0, mb * 2 * BM + rank * BM, lbar);
                    issue_raw();
                    if (++s == S) { s = 0; ph ^= 1; }
                    continue;
                }
                if (rank == 0) mbar_expect_tx(full_bar(s), 2 * Cfg::STAGE + (Q8 ? 16 : 0));
                tma_load_2d_pair(sa, ma, k0, mb * 2 * BM + rank * BM, lbar);
                if (B_MN) {
#pragma unroll
                    for (int j = 0; j < BH2 / 64; ++j) tma_load_2d_pair(sb + j * 8192, mbm, n0 + 64 * j, k0, lbar);
                } else {
                    tma_load_2d_pair(sb, mbm, k0, n0, lbar);
                }
                if (++s == S) { s = 0; ph ^= 1; }
            }
        }
        // no quants may still be landing when the CTA leaves (after a failed wait, the converters
        // stop early): the latest load of each slot is waited for, bounded and regardless of the
        // error word; on the normal path those phases completed long ago
        if (Q8)
            for (int i = raw_issued - 1; i >= 0 && i >= raw_issued - R; --i)
                mbar_wait_drain(raw_bar(i % R), (uint32_t)((i / R) & 1));
        if (SK && ok && role == SK_PART_IN) {
            // The last item is the head of a split tile: once the next pair has published the
            // tile's tail (its first item), stream this CTA's 128 KB of it into the next four
            // stages of the ring as the mainloop releases them.
            if (BN2 == 256) {
                int* flag = p.sk_flag + (pair + 1) * 2 + (int)rank;
                if (flag_wait(flag, Cfg::EW, p.err, 18)) {
                    *flag = 0;  // consumed; the next launch starts from zero
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                    mbar_expect_tx(part_bar, SK_CTA_BYTES);
                    const unsigned char* src = reinterpret_cast<const unsigned char*>(
                        p.sk_part + ((size_t)(pair + 1) * 2 + rank) * SK_CTA_FLOATS);
                    for (int j = 0; j < SK_CTA_BYTES / Cfg::STAGE; ++j) {
                        if (!mbar_wait(empty_bar(s), ph ^ 1, p.err, 11)) break;
                        bulk_load(base + s * Cfg::STAGE, src + (size_t)j * Cfg::STAGE, Cfg::STAGE, part_bar);
                        if (++s == S) { s = 0; ph ^= 1; }
                    }
                } else {
                    mbar_arrive(part_bar);  // no data: let the epilogue go on (the error is recorded)
                }
                mbar_wait(part_bar, 0, p.err, 19);  // no copy still in flight when the CTA exits
            }
        }
    } else if (warp == 1 && lane == 0 && rank == 0) {
        // ------------------------------------------------------------ MMA issuer (leader)
        const uint32_t idesc = IDESC_F16_F32ACC | ((B_MN ? 1u : 0u) << 16) |
                               ((uint32_t)(BN2 >> 3) << 17) | ((uint32_t)((2 * BM) >> 4) << 24);
        const uint64_t a_desc0 = smem_desc(base, 16, 1024);
        const uint64_t b_desc0 = B_MN ? smem_desc(base + Cfg::A_BYTES, 8192, 1024)
                                      : smem_desc(base + Cfg::A_BYTES, 16, 1024);
        constexpr uint32_t A_STEP = 32 >> 4, B_STEP = (B_MN ? 2048 : 32) >> 4;
        const uint32_t empty0 = map_rank(empty_bar(0), 0), empty1 = map_rank(empty_bar(0), 1);
        int s = 0, u = 0;
        uint32_t ph = 0;
        bool ok = true;
        PairWork w(SK ? 1 : 0, nk, ntiles, pair, npairs);
        int tile, kb0, kb1, role;
        for (; ok && w.next(tile, kb0, kb1, role); ++u) {
            const int a = u & 1;
            ok = mbar_wait(tempty_bar(a), ((u >> 1) & 1) ^ 1, p.err, 12);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t tacc = tmem_base + a * BN2;
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(full_bar(s), ph, p.err, 13)) { ok = false; break; }
                const uint64_t soff = (uint64_t)((s * Cfg::STAGE) >> 4);
                const uint64_t ad = a_desc0 + soff, bd = b_desc0 + soff;
                const int kv = kb >= nk1 ? p.K2 - (kb - nk1) * BKE : BKE;
                if (kv >= BKE) {
#pragma unroll
                    for (int k16 = 0; k16 < BKE / 16; ++k16)
                        mma_f16_pair(tacc, ad + A_STEP * k16, bd + B_STEP * k16, idesc, (kb > kb0 || k16) ? 1u : 0u);
                } else {
                    for (int k16 = 0; k16 < (kv + 15) / 16; ++k16)
                        mma_f16_pair(tacc, ad + A_STEP * k16, bd + B_STEP * k16, idesc, (kb > kb0 || k16) ? 1u : 0u);
                }
                mma_commit_pair(empty0 + 8 * s);
                mma_commit_pair(empty1 + 8 * s);
                if (++s == S) { s = 0; ph ^= 1; }
            }
            if (!ok) break;
            mma_commit_pair(map_rank(tfull_bar(a), 0));
            mma_commit_pair(map_rank(tfull_bar(a), 1));
        }
        mma_commit_pair(map_rank(drain_bar, 0));
        mbar_wait(drain_bar, 0, p.err, 16);
    } else if (Q8 && warp >= 2 + Cfg::EW) {
        // ------------------------------------------------------------ Q8_0 converters (both CTAs)
        // Same k-block schedule as the producer.  Per k-block: wait until the stage is free, wait
        // for its raw slot (Q8_0 segments), write the f16 operand tile, make it visible to the
        // tensor core (async proxy), and count this CTA into the leader's full barrier: a local
        // arrival in the leader, a 16-byte DSMEM copy with complete_tx from the peer (an
        // asynchronous signal: the converters go on while it travels).  The producer keeps the
        // raw ring filled ahead of them.
        // Two groups of converter warps take alternate k-blocks, so one group's shared-memory
        // latency, fence and barrier overlap the other's conversion.
        constexpr int CT = (Cfg::CW ? Cfg::CW : 2) * 32;  // converter threads (the non-Q8 kernel has none)
        constexpr int GT = CT / 2;                          // threads per group
        const int ct = threadIdx.x - (2 + Cfg::EW) * 32;
        const int grp = ct / GT, gct = ct % GT;
        const uint32_t leader_full0 = map_rank(full_bar(0), 0);
        const uint32_t sig_local = bars + SIG_OFF, sig_leader = map_rank(bars + SIG_OFF, 0);
        int s = 0, r = 0, seq = 0;
        uint32_t ph = 0, rph = 0;  // operand-ring parity, raw-ring parity
        PairWork w(SK ? 1 : 0, nk, ntiles, pair, npairs);
        int tile, kb0, kb1, role;
        bool ok = true;
        while (ok && w.next(tile, kb0, kb1, role)) {
            for (int kb = kb0; kb < kb1; ++kb, ++seq) {
                const bool conv = (p.q8mask >> (kb >= nk1 ? 1 : 0)) & 1;
                if ((seq & 1) == grp) {
                    bool got = mbar_wait(empty_bar(s), ph ^ 1, p.err, 22);
                    if (conv && got) {
                        got = mbar_wait(raw_bar(r), rph, p.err, 21);
                        if (got) {
                            convert_q8_stage<BH2, B_MN, GT>(smem, raw_off + r * Cfg::RAW,
                                                            s * Cfg::STAGE + Cfg::A_BYTES, gct);
                            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        }
                    }
                    // the group's threads agree (and have written the tile) before the signal; on
                    // a failed wait they leave together (the MMA then gives up on its own bounded
                    // wait, and the other group on its own)
                    uint32_t all;
                    asm volatile(
                        "{\n\t.reg .pred p, q;\n\t"
                        "setp.ne.u32 p, %1, 0;\n\t"
                        "bar.red.and.pred q, %2, %3, p;\n\t"
                        "selp.u32 %0, 1, 0, q;\n\t}"
                        : "=r"(all)
                        : "r"(got ? 1u : 0u), "r"(1 + grp), "n"(GT)
                        : "memory");
                    if (!all) {
                        ok = false;
                        break;
                    }
                    if (gct == 0) {
                        if (rank == 0) {
                            mbar_arrive(full_bar(s));
                        } else {
                            asm volatile(
                                "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], 16, [%2];"
                                ::"r"(sig_leader), "r"(sig_local), "r"(leader_full0 + 8 * s)
                                : "memory");
                        }
                    }
                }
                if (conv && ++r == R) { r = 0; rph ^= 1; }
                if (++s == S) { s = 0; ph ^= 1; }
            }
        }
    } else if (warp >= 2) {
        // ------------------------------------------------------------ epilogue (both CTAs)
        // TMEM lanes 32*quad .. 32*quad+31, columns coff .. coff + WCOLS - 1 of the tile
        constexpr int WCOLS = BN2 / (Cfg::EW / 4);  // columns per epilogue warp
        constexpr int WARP_FLOATS = 32 * WCOLS;     // its share of a stream-K partial
        const int ew = warp - 2, quad = warp & 3, coff = (ew >> 2) * WCOLS;
        EpiTiles tiles;
        tiles.o = smem + S * Cfg::STAGE + ew * EPI_OUT_BYTES;
        tiles.x = smem + S * Cfg::STAGE + Cfg::EW * EPI_OUT_BYTES + ew * EPI_AUX_BYTES;
        tiles.o_s = smem_u32(tiles.o);
        tiles.x_s = smem_u32(tiles.x);
        const uint32_t leader_tempty0 = map_rank(tempty_bar(0), 0), leader_tempty1 = map_rank(tempty_bar(1), 0);
        const int mlim = min(p.M, p.mvalid);
        auto tile_rows = [&](int tl, int& m_base, int& rows, int& n0) {
            m_base = (tl % num_m2) * 2 * BM + (int)rank * BM + quad * 32;
            rows = tl < ntiles ? max(0, min(32, mlim - m_base)) : 0;
            n0 = (tl / num_m2) * BN2 + coff;
        };
        PairWork w(SK ? 1 : 0, nk, ntiles, pair, npairs);
        // the ring slot after this pair's last k-block: where a stream-K partial lands
        int units = 0, first_epi = pair;
        if (SK) {
            first_epi = ntiles;
            PairWork c = w;
            int t, k0, k1, r;
            while (c.next(t, k0, k1, r)) {
                units += k1 - k0;
                if (r != SK_PART_OUT && first_epi == ntiles) first_epi = t;
            }
        }
        float4 pre[8];
        {
            int mb0, r0, n00;
            tile_rows(first_epi, mb0, r0, n00);
            fetch_input(p, epi_input_kind(p), mb0, r0, n00, lane, pre);
        }
        int tile, kb0, kb1, role;
        bool have = w.next(tile, kb0, kb1, role);
        for (int u = 0; have; ++u) {
            int ntile = ntiles, nkb0, nkb1, nrole;
            const bool nhave = w.next(ntile, nkb0, nkb1, nrole);
            if (!nhave) ntile = ntiles;
            const int a = u & 1;
            bool ok = true;
            if (lane == 0) ok = mbar_wait(tfull_bar(a), (u >> 1) & 1, p.err, 14);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t trow = tmem_base + ((uint32_t)(quad * 32) << 16) + a * BN2 + coff;
            if (SK && role == SK_PART_OUT) {
                // tail of a split tile: raw fp32 accumulators to slot `pair`, then count this warp in
                float4* dst = reinterpret_cast<float4*>(p.sk_part + ((size_t)pair * 2 + rank) * SK_CTA_FLOATS +
                                                        (size_t)ew * WARP_FLOATS);
                for (int c = 0; c < WCOLS / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(trow + c * 32, r);
#pragma unroll
                    for (int g = 0; g < 8; ++g)
                        __stcg(dst + (c * 8 + g) * 32 + lane,
                               make_float4(__uint_as_float(r[4 * g]), __uint_as_float(r[4 * g + 1]),
                                           __uint_as_float(r[4 * g + 2]), __uint_as_float(r[4 * g + 3])));
                }
                __threadfence();
                __syncwarp();
                if (lane == 0) red_release_add(p.sk_flag + pair * 2 + (int)rank, 1);
            } else {
                const float4* part = nullptr;
                if (SK && role == SK_PART_IN && BN2 == 256) {
                    // head of a split tile: the producer streams the tail's partial into the ring
                    mbar_wait(part_bar, 0, p.err, 20);
                    const int at = ew * WARP_FLOATS * 4;  // this warp's bytes in the streamed partial
                    part = reinterpret_cast<const float4*>(smem + ((units + at / Cfg::STAGE) % S) * Cfg::STAGE +
                                                           at % Cfg::STAGE);
                }
                int m_base, rows, n0, nm, nr, nn;
                tile_rows(tile, m_base, rows, n0);
                tile_rows(ntile, nm, nr, nn);
                epilogue_tile<WCOLS / 32>(p, maps, trow, m_base, rows, n0, nm, nr, nn, tiles, lane, pre, part);
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(a ? leader_tempty1 : leader_tempty0);
            tile = ntile; kb0 = nkb0; kb1 = nkb1; role = nrole; have = nhave;
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    cluster_sync();  // no CTA leaves while its partner may still signal it or read its smem
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    __syncwarp();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(Cfg::TMEM_COLS));
}

// ---------------------------------------------------------------------------------------
// host side: tensor maps through the driver entry point (no libcuda link dependency)

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !p)
            throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
        fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2D f16 row-major tensor [rows][cols] with row stride ld (elements); box {box_cols, box_rows}.
void make_map(CUtensorMap* map, const f16* ptr, long rows, long cols, long ld, int box_cols, int box_rows) {
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (ld * 2) % 16)
        throw std::runtime_error("gemm_tc: operand not 16-byte aligned");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<f16*>(ptr), dims, strides, box,
                             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
}

// Raw (unswizzled) maps of a Q8_0 weight view: quants [rows][cols] (row stride ld bytes) and f16
// scales [rows][cols] (row stride ld elements).
void make_map_raw(CUtensorMap* map, const void* ptr, bool f16v, long rows, long cols, long ld, int box_cols,
                  int box_rows) {
    const int esz = f16v ? 2 : 1;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (ld * esz) % 16 || (box_cols * esz) % 16)
        throw std::runtime_error("gemm_tc: Q8_0 operand not 16-byte aligned");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * esz};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(map, f16v ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                             const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (Q8_0) failed: " + std::to_string((int)r));
}

// B segment maps: f16 (128-byte swizzle, straight into the operand tile) or Q8_0 (quants and
// scales into the raw ring).  K-major B is [N][K], MN-major [K][N]; bh = B rows per CTA.
void make_b_maps(CUtensorMap* bmap, CUtensorMap* smap, const f16* B, const uint8_t* Bq, const f16* Bd, long ldb,
                 long ldd, int K, int N, bool mn, int bh) {
    if (!Bq) {
        if (mn) make_map(bmap, B, K, N, ldb, 64, BKE);
        else make_map(bmap, B, N, K, ldb, BKE, bh);
        *smap = *bmap;
        return;
    }
    if (mn) {
        make_map_raw(bmap, Bq, false, K, N, ldb, bh, BKE);          // bh quants (n) x 64 rows (k)
        make_map_raw(smap, Bd, true, N / 32, K, ldd, BKE, bh / 32);  // 64 scales (k) x bh / 32 rows
    } else {
        make_map_raw(bmap, Bq, false, N, K, ldb, BKE, bh);          // 64 quants (k) x bh rows (n)
        make_map_raw(smap, Bd, true, K / 32, N, ldd, bh, 2);         // bh scales (n) x 2 rows (k / 32)
    }
}

// Epilogue store maps: the output as fp32 (box 32 x 32, 128-byte swizzle) or f16 (box 32 x 32,
// 64-byte swizzle) over rows min(M, mvalid); the f16 side output (aux) the same way.
void make_store_map(CUtensorMap* map, const void* ptr, bool f32, long rows, long cols, long ld) {
    const int esz = f32 ? 4 : 2;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (ld * esz) % 16)
        throw std::runtime_error("gemm_tc: epilogue output not 16-byte aligned");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * esz)};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                             const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (store) failed: " + std::to_string((int)r));
}

// rows of A in memory: the maps end there and TMA reads the rows past them as zero
long a_rows(const GemmArgs& a) { return a.arows > 0 && a.arows < a.M ? a.arows : a.M; }

void make_epilogue_maps(TcMaps& maps, const GemmArgs& a) {
    const long rows = a.M < a.mvalid ? a.M : a.mvalid;
    const bool f32 = a.mode == EPI_STORE_F32 || a.mode == EPI_ACCUM_F32 || a.mode == EPI_RESID_F32;
    make_store_map(&maps.out, a.out, f32, rows, a.N, a.ldo);
    if (a.aux) make_store_map(&maps.aux, a.aux, false, rows, a.N, a.ldaux);
    else maps.aux = maps.out;
    if (a.out_h && f32) make_store_map(&maps.out_h, a.out_h, false, rows, a.N, a.ldo);
    else maps.out_h = maps.out;
}


template <int BN, bool B_MN>
void launch_tc(const GemmArgs& a, int* err, cudaStream_t s) {
    using Cfg = TcCfg<BN>;
    TcMaps maps;
    // A: [M][K] K-major; box 64 (k) x 128 (m)
    make_map(&maps.a1, a.A1, a_rows(a), a.K1, a.lda1, BKE, BM);
    if (B_MN) make_map(&maps.b1, a.B1, a.K1, a.N, a.ldb1, 64, BKE);   // [K][N]: box 64 (n) x 64 (k)
    else make_map(&maps.b1, a.B1, a.N, a.K1, a.ldb1, BKE, BN);        // [N][K]: box 64 (k) x BN (n)
    if (a.K2 > 0) {
        make_map(&maps.a2, a.A2, a_rows(a), a.K2, a.lda2, BKE, BM);
        if (B_MN) make_map(&maps.b2, a.B2, a.K2, a.N, a.ldb2, 64, BKE);
        else make_map(&maps.b2, a.B2, a.N, a.K2, a.ldb2, BKE, BN);
    } else {
        maps.a2 = maps.a1;
        maps.b2 = maps.b1;
    }
    make_epilogue_maps(maps, a);
    TcParams p;
    p.M = a.M; p.N = a.N; p.K1 = a.K1; p.K2 = a.K2;
    p.num_m = (a.M + BM - 1) / BM; p.num_n = a.N / BN;
    p.q8mask = 0; p.late_wait = 0; p.sk_part = nullptr; p.sk_flag = nullptr;
    p.mode = a.mode; p.alpha = a.alpha; p.colscale = a.colscale; p.out = a.out; p.ldo = a.ldo;
    p.resid = a.resid; p.ldr = a.ldr; p.aux = a.aux; p.ldaux = a.ldaux; p.auxin = a.auxin; p.ldauxin = a.ldauxin;
    p.colscale2 = a.colscale2; p.bias = a.bias; p.nvalid = a.nvalid; p.mvalid = a.mvalid; p.err = err;
    p.rope = a.rope; p.rope_T = a.rope_T; p.rope_cols = a.rope_cols;
    p.out_h = (a.mode == EPI_STORE_F32 || a.mode == EPI_ACCUM_F32 || a.mode == EPI_RESID_F32) ? a.out_h : nullptr;
    auto kern = gemm_tc_kernel<BN, B_MN>;
    static DeviceOnce once;
    once([&] { cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM); });
    const int num_sms = current_sm_count();
    const int tiles = p.num_m * p.num_n;
    const int grid = tiles < num_sms ? tiles : num_sms;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(NTHREADS, 1, 1);
    cfg.dynamicSmemBytes = Cfg::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    pdl_attr(attr[0]);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, maps, p);
}

// Stream-K where it pays: 256-wide pair tiles, at least as many tiles as pairs (one split per
// tile at most) and a workspace.  Its cost is the pair's share of k-blocks plus the partial
// tile's round trip through L2 (a 256 KB write early, a read at the end, both while every SM
// streams operands), measured at about 12 k-blocks of 256 x 256 x 64; whole tiles cost their
// rounds.  So only long reductions with an idle last round gain (K = 3072, 4096 at N = 1024).
bool sk_pays(int bn2, int tiles, int pairs, const GemmArgs& a) {
    if (bn2 != 256 || !a.sk_part || !a.sk_flag || tiles < pairs || pairs < 2) return false;
    const long nk = (a.K1 + BKE - 1) / BKE + (a.K2 + BKE - 1) / BKE;
    const long rounds = (tiles + pairs - 1) / pairs;
    const long share = (tiles * nk + pairs - 1) / pairs;
    return share + 12 < 0.92 * rounds * nk;
}

template <int BN2, bool B_MN, bool Q8>
void launch_tc2(const GemmArgs& a, int* err, cudaStream_t s) {
    using Cfg = Tc2Cfg<BN2, Q8>;
    constexpr int BH2 = Cfg::BH;
    TcMaps maps;
    make_map(&maps.a1, a.A1, a_rows(a), a.K1, a.lda1, BKE, BM);
    make_b_maps(&maps.b1, &maps.s1, a.B1, a.B1q, a.B1d, a.ldb1, a.ldd1, a.K1, a.N, B_MN, BH2);
    if (a.K2 > 0) {
        make_map(&maps.a2, a.A2, a_rows(a), a.K2, a.lda2, BKE, BM);
        make_b_maps(&maps.b2, &maps.s2, a.B2, a.B2q, a.B2d, a.ldb2, a.ldd2, a.K2, a.N, B_MN, BH2);
    } else {
        maps.a2 = maps.a1;
        maps.b2 = maps.b1;
        maps.s2 = maps.s1;
    }
    make_epilogue_maps(maps, a);
    TcParams p;
    p.M = a.M; p.N = a.N; p.K1 = a.K1; p.K2 = a.K2;
    p.num_m = (a.M + BM - 1) / BM; p.num_n = a.N / BN2;
    p.mode = a.mode; p.alpha = a.alpha; p.colscale = a.colscale; p.out = a.out; p.ldo = a.ldo;
    p.resid = a.resid; p.ldr = a.ldr; p.aux = a.aux; p.ldaux = a.ldaux; p.auxin = a.auxin; p.ldauxin = a.ldauxin;
    p.colscale2 = a.colscale2; p.bias = a.bias; p.nvalid = a.nvalid; p.mvalid = a.mvalid; p.err = err;
    p.rope = a.rope; p.rope_T = a.rope_T; p.rope_cols = a.rope_cols;
    p.out_h = (a.mode == EPI_STORE_F32 || a.mode == EPI_ACCUM_F32 || a.mode == EPI_RESID_F32) ? a.out_h : nullptr;
    p.sk_part = a.sk_part; p.sk_flag = a.sk_flag;
    p.q8mask = (a.B1q ? 1 : 0) | (a.K2 > 0 && a.B2q ? 2 : 0);
    p.late_wait = a.a2_from_prev && a.K2 > 0 ? 1 : 0;
    auto whole = gemm_tc2_kernel<BN2, B_MN, false, Q8>;
    auto split = gemm_tc2_kernel<BN2, B_MN, BN2 == 256, Q8>;
    static DeviceOnce once;
    once([&] {
        for (auto k : {whole, split}) {
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
            cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
        }
    });
    const int num_sms = current_sm_count();
    const int tiles = ((a.M + 2 * BM - 1) / (2 * BM)) * (a.N / BN2);
    const int pairs = tiles < num_sms / 2 ? tiles : num_sms / 2;
    const bool use_split = sk_pays(BN2, tiles, pairs, a);
    const auto kern = use_split ? split : whole;
    // stream-K: a pair whose range holds only the head of a tile (no A2 k-blocks) would store
    // outputs without having waited, so the early start is for whole tiles only
    if (use_split) p.late_wait = 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
    cfg.dynamicSmemBytes = Cfg::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    pdl_attr(attr[1]);
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaLaunchKernelEx(&cfg, kern, maps, p);
}

}  // namespace

namespace {
bool q8_args(const GemmArgs& a) { return a.B1q || (a.K2 > 0 && a.B2q); }
bool q8_segment_ok(const uint8_t* q, const f16* d, long ldq, long ldd, int K) {
    const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(d);
    return d && (al & 15) == 0 && ldq % 16 == 0 && (ldd * 2) % 16 == 0 && K % BKE == 0;
}
}  // namespace

bool gemm_tc_supported(const GemmArgs& a) {
    if (!a.a_kmajor) return false;
    if (a.M < BM || a.N % 128 || a.K1 % BKE || a.K1 <= 0 || a.splitk != 1) return false;
    if (a.K2 && (a.K2 % 8 || !a.A2 || !(a.B2 || a.B2q))) return false;
    // Q8_0 weights: the 2-CTA kernel only (it has the converter warps)
    if (q8_args(a) && (a.M <= BM || (a.B1q && !q8_segment_ok(a.B1q, a.B1d, a.ldb1, a.ldd1, a.K1)) ||
                       (a.K2 > 0 && a.B2q && !q8_segment_ok(a.B2q, a.B2d, a.ldb2, a.ldd2, a.K2))))
        return false;
    // rows past mvalid are clipped by the store maps and skipped by the epilogue's inputs
    if (a.mode == EPI_ATOMIC_F32 || a.nvalid < a.N || a.mvalid <= 0) return false;
    if ((a.mode == EPI_GELU_BWD || a.mode == EPI_GELU_BWD_D) && a.aux)
        return false;  // its pre-activation input occupies the side tile
    if (a.ldo % 8 || (a.aux && a.ldaux % 8) || (a.auxin && a.ldauxin % 8) || (a.resid && a.ldr % 4)) return false;
    const uintptr_t al = reinterpret_cast<uintptr_t>(a.out) | reinterpret_cast<uintptr_t>(a.aux) |
                         reinterpret_cast<uintptr_t>(a.auxin) | reinterpret_cast<uintptr_t>(a.resid) |
                         reinterpret_cast<uintptr_t>(a.colscale) | reinterpret_cast<uintptr_t>(a.A1) |
                         reinterpret_cast<uintptr_t>(a.B1) | reinterpret_cast<uintptr_t>(a.A2) |
                         reinterpret_cast<uintptr_t>(a.B2) | reinterpret_cast<uintptr_t>(a.out_h);
    return (al & 15) == 0;
}

bool gemm_tc2_supported(const GemmArgs& a) { return gemm_tc_supported(a) && a.M > BM; }

void gemm_tc2_width(const GemmArgs& a, int* err, cudaStream_t s, int width) {
    const bool q8 = q8_args(a);
    if (width == 256) {
        if (a.b_kmajor) q8 ? launch_tc2<256, false, true>(a, err, s) : launch_tc2<256, false, false>(a, err, s);
        else q8 ? launch_tc2<256, true, true>(a, err, s) : launch_tc2<256, true, false>(a, err, s);
    } else {
        if (a.b_kmajor) q8 ? launch_tc2<128, false, true>(a, err, s) : launch_tc2<128, false, false>(a, err, s);
        else q8 ? launch_tc2<128, true, true>(a, err, s) : launch_tc2<128, true, false>(a, err, s);
    }
}

long gemm_sk_part_floats(int num_sms) { return (long)(num_sms / 2) * 2 * SK_CTA_FLOATS; }
int gemm_sk_flag_count(int num_sms) { return (num_sms / 2) * 2; }

void gemm_tc2(const GemmArgs& a, int* err, cudaStream_t s) { gemm_tc2_width(a, err, s, a.N % 256 == 0 ? 256 : 128); }

void gemm_tc_auto(const GemmArgs& a, int* err, cudaStream_t s) {
    const int num_sms = current_sm_count();
    // Each SM computes 128-row tiles in every variant; the cost of a launch is its number of
    // rounds over the SMs times the tile width, scaled by per-column efficiencies measured on
    // the cfg-2 shapes (256-wide 2-CTA tiles fastest; 128-wide pair tiles 1.6x slower per
    // column, so they only win where they save whole rounds).
    static const double eff[3] = {1.05, 1.0, 1.62};  // 1-CTA 256 (or 128), 2-CTA 256, 2-CTA 128
    auto rounds = [&](long tiles, long slots) { return (tiles + slots - 1) / slots; };
    const long m1 = (a.M + BM - 1) / BM, m2 = (a.M + 2 * BM - 1) / (2 * BM), pairs = num_sms / 2;
    const int w1 = a.N % 256 == 0 ? 256 : 128;
    double best = q8_args(a) ? 1e30 : rounds(m1 * (a.N / w1), num_sms) * (double)w1 * eff[0];
    int choice = 0;
    if (gemm_tc2_supported(a)) {
        if (a.N % 256 == 0) {
            const long t2 = m2 * (a.N / 256);
            // stream-K spreads the k-blocks evenly: cost by the mean share plus its fix-up
            const long nk = (a.K1 + BKE - 1) / BKE + (a.K2 + BKE - 1) / BKE;
            const double c = sk_pays(256, (int)t2, (int)std::min(t2, pairs), a)
                                 ? ((double)t2 * nk / pairs + 12.0) / nk * 256.0 * eff[1]
                                 : rounds(t2, pairs) * 256.0 * eff[1];
            if (c < best) { best = c; choice = 1; }
        }
        const double c = rounds(m2 * (a.N / 128), pairs) * 128.0 * eff[2];
        if (c < best) { best = c; choice = 2; }
    }
    if (choice == 0) gemm_tc(a, err, s);
    else gemm_tc2_width(a, err, s, choice == 1 ? 256 : 128);
}

void gemm_tc(const GemmArgs& a, int* err, cudaStream_t s) {
    if (q8_args(a)) throw std::runtime_error("gemm_tc: Q8_0 weights need the 2-CTA kernel");
    const long tiles256 = (long)((a.M + BM - 1) / BM) * (a.N / 256);
    static const int force_bn = [] {
        const char* e = std::getenv("ACTRAIN_TC_BN");  // tuning experiments only
        return e ? std::atoi(e) : 0;
    }();
    // 256-wide tiles whenever N allows: measured faster than 128-wide at every cfg-2 shape,
    // even when they leave part of the last wave idle (higher FLOP per byte staged from L2)
    (void)tiles256;
    const bool wide = a.N % 256 == 0 && force_bn != 128;
    if (a.b_kmajor) {
        if (wide) launch_tc<256, false>(a, err, s);
        else launch_tc<128, false>(a, err, s);
    } else {
        if (wide) launch_tc<256, true>(a, err, s);
        else launch_tc<128, true>(a, err, s);
    }
}

void tc_make_map(CUtensorMap* map, const f16* ptr, long rows, long cols, long ld, int box_cols, int box_rows) {
    make_map(map, ptr, rows, cols, ld, box_cols, box_rows);
}

void tc_make_map_raw(CUtensorMap* map, const void* ptr, bool f16v, long rows, long cols, long ld, int box_cols,
                     int box_rows) {
    make_map_raw(map, ptr, f16v, rows, cols, ld, box_cols, box_rows);
}

void tc_make_map3(CUtensorMap* map, const f16* ptr, long clips, long rows, long cols, long ld, int box_cols,
                  int box_rows) {
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (ld * 2) % 16)
        throw std::runtime_error("tc_make_map3: operand not 16-byte aligned");
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)clips};
    cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)(rows * ld * 2)};
    cuuint32_t box[3] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<f16*>(ptr), dims, strides, box,
                             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (3-D) failed: " + std::to_string((int)r));
}

}  // namespace act
