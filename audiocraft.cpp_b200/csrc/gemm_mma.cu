// gemm_mma.cu -- generic f16 GEMM on the warp-level tensor-core path (mma.sync m16n8k16).
//
// Covers every operand layout the training step needs (forward Y = X W^T, input gradient
// dX = dY W, adapter gradients dB = dY^T U and dA = dU^T X), a second K segment for the
// LoRA rank block, split-K for the token reductions, and the fused epilogues.  The dense
// projections of the big configurations go through the tcgen05 kernel in gemm_tc.cu; this
// kernel is the fallback shape-wise (skinny, transposed, split-K) and the cross-check.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <stdexcept>

namespace act {

namespace {

template <int BM, int BN, bool AK, bool BKM, int BK, int STAGES>
struct Smem {
    // K-major tile: [rows][BK + 8]; MN-major tile: [BK][cols + 8]
    static constexpr int A_ELEMS = AK ? BM * (BK + 8) : BK * (BM + 8);
    static constexpr int B_ELEMS = BKM ? BN * (BK + 8) : BK * (BN + 8);
    static constexpr int STAGE = A_ELEMS + B_ELEMS;
    static constexpr int BYTES = STAGE * STAGES * 2;
};

template <int BM, int BN, int WM_, int WN_, bool AK, bool BKM, int BK, int STAGES>
__global__ void __launch_bounds__(WM_* WN_ * 32)
gemm_mma_kernel(const GemmArgs p) {
    pdl_wait();
    pdl_trigger();
    constexpr int NT = WM_ * WN_ * 32;
    constexpr int WTM = BM / WM_, WTN = BN / WN_;
    constexpr int MI = WTM / 16, NI = WTN / 8;
    static_assert(NI % 2 == 0, "warp tile N must be a multiple of 16");
    using S = Smem<BM, BN, AK, BKM, BK, STAGES>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    f16* smem = reinterpret_cast<f16*>(smem_raw);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = warp / WN_, wn = warp % WN_;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;

    const int kt1 = (p.K1 + BK - 1) / BK, kt2 = (p.K2 + BK - 1) / BK, ktot = kt1 + kt2;
    const int per = (ktot + p.splitk - 1) / p.splitk;
    const int kbeg = blockIdx.z * per, kend = min(ktot, kbeg + per);
    const int ntiles = max(0, kend - kbeg);

    auto load_tile = [&](int t, int stage) {
        const int kt = kbeg + t;
        const bool seg2 = kt >= kt1;
        const f16* A = seg2 ? p.A2 : p.A1;
        const f16* B = seg2 ? p.B2 : p.B1;
        const long lda = seg2 ? p.lda2 : p.lda1, ldb = seg2 ? p.ldb2 : p.ldb1;
        const int Kseg = seg2 ? p.K2 : p.K1;
        const int k0 = (seg2 ? kt - kt1 : kt) * BK;
        f16* sA = smem + stage * S::STAGE;
        f16* sB = sA + S::A_ELEMS;
        if (AK) {
            for (int c = tid; c < BM * (BK / 8); c += NT) {
                const int r = c / (BK / 8), kc = (c % (BK / 8)) * 8;
                const int gm = m0 + r, gk = k0 + kc;
                const bool ok = gm < p.M && gk < Kseg;
                cp_async16(sA + r * (BK + 8) + kc, ok ? A + (long)gm * lda + gk : A, ok);
            }
        } else {
            for (int c = tid; c < BK * (BM / 8); c += NT) {
                const int kr = c / (BM / 8), mc = (c % (BM / 8)) * 8;
                const int gm = m0 + mc, gk = k0 + kr;
                const bool ok = gm < p.M && gk < Kseg;
                cp_async16(sA + kr * (BM + 8) + mc, ok ? A + (long)gk * lda + gm : A, ok);
            }
        }
        if (BKM) {
            for (int c = tid; c < BN * (BK / 8); c += NT) {
                const int r = c / (BK / 8), kc = (c % (BK / 8)) * 8;
                const int gn = n0 + r, gk = k0 + kc;
                const bool ok = gn < p.N && gk < Kseg;
                cp_async16(sB + r * (BK + 8) + kc, ok ? B + (long)gn * ldb + gk : B, ok);
            }
        } else {
            for (int c = tid; c < BK * (BN / 8); c += NT) {
                const int kr = c / (BN / 8), nc = (c % (BN / 8)) * 8;
                const int gn = n0 + nc, gk = k0 + kr;
                const bool ok = gn < p.N && gk < Kseg;
                cp_async16(sB + kr * (BN + 8) + nc, ok ? B + (long)gk * ldb + gn : B, ok);
            }
        }
    };

    float acc[MI][NI][4];
#pragma unroll
    for (int i = 0; i < MI; ++i)
#pragma unroll
        for (int j = 0; j < NI; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;

#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
        if (s < ntiles) load_tile(s, s);
        cp_async_commit();
    }

    const int lr = lane & 7, lsel = lane >> 3;
    for (int t = 0; t < ntiles; ++t) {
        cp_async_wait<STAGES - 2>();
        __syncthreads();
        if (t + STAGES - 1 < ntiles) load_tile(t + STAGES - 1, (t + STAGES - 1) % STAGES);
        cp_async_commit();
        const f16* sA = smem + (t % STAGES) * S::STAGE;
        const f16* sB = sA + S::A_ELEMS;
#pragma unroll
        for (int kk = 0; kk < BK; kk += 16) {
            uint32_t af[MI][4];
#pragma unroll
            for (int mi = 0; mi < MI; ++mi) {
                const int mb = wm * WTM + mi * 16;
                if (AK) {
                    const f16* ptr = sA + (mb + lr + 8 * (lsel & 1)) * (BK + 8) + kk + 8 * (lsel >> 1);
                    ldsm_x4(af[mi][0], af[mi][1], af[mi][2], af[mi][3], ptr);
                } else {
                    const f16* ptr = sA + (kk + lr + 8 * (lsel >> 1)) * (BM + 8) + mb + 8 * (lsel & 1);
                    ldsm_x4_t(af[mi][0], af[mi][1], af[mi][2], af[mi][3], ptr);
                }
            }
#pragma unroll
            for (int nj = 0; nj < NI / 2; ++nj) {
                const int nb = wn * WTN + nj * 16;
                uint32_t b0, b1, b2, b3;
                if (BKM) {
                    const f16* ptr = sB + (nb + lr + 8 * (lsel >> 1)) * (BK + 8) + kk + 8 * (lsel & 1);
                    ldsm_x4(b0, b1, b2, b3, ptr);
                } else {
                    const f16* ptr = sB + (kk + lr + 8 * (lsel & 1)) * (BN + 8) + nb + 8 * (lsel >> 1);
                    ldsm_x4_t(b0, b1, b2, b3, ptr);
                }
#pragma unroll
                for (int mi = 0; mi < MI; ++mi) {
                    mma_sync_f16(acc[mi][2 * nj], af[mi], b0, b1);
                    mma_sync_f16(acc[mi][2 * nj + 1], af[mi], b2, b3);
                }
            }
        }
    }
    cp_async_wait<0>();

    // ---------------- epilogue ----------------
    const int g = lane >> 2, q = lane & 3;
#pragma unroll
    for (int mi = 0; mi < MI; ++mi)
#pragma unroll
        for (int ni = 0; ni < NI; ++ni)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int m = m0 + wm * WTM + mi * 16 + g + 8 * h;
                const int n = n0 + wn * WTN + ni * 8 + 2 * q;
                if (m >= p.M || m >= p.mvalid || n >= p.N || n >= p.nvalid) continue;
                const bool two = (n + 1 < p.N) && (n + 1 < p.nvalid);
                float v0 = acc[mi][ni][2 * h] * p.alpha, v1 = acc[mi][ni][2 * h + 1] * p.alpha;
                if (p.colscale) {
                    v0 *= p.colscale[n];
                    if (two) v1 *= p.colscale[n + 1];
                }
                if (p.aux && p.mode != EPI_GELU) {
                    f16* a = p.aux + (long)m * p.ldaux + n;
                    if (two) *reinterpret_cast<uint32_t*>(a) = pack_f16(v0, v1);
                    else a[0] = __float2half_rn(v0);
                }
                if (p.rope && n < p.rope_cols) {  // n is even: (v0, v1) is one rotary pair
                    const float2 t = reinterpret_cast<const float2*>(p.rope)[(long)(m % p.rope_T) * 32 + (n % 64) / 2];
                    const float x0 = v0, x1 = v1;
                    v0 = x0 * t.x - x1 * t.y;
                    v1 = x0 * t.y + x1 * t.x;
                }
                switch (p.mode) {
                    case EPI_STORE_F32:
                    case EPI_ACCUM_F32:
                    case EPI_RESID_F32: {
                        float* o = static_cast<float*>(p.out) + (long)m * p.ldo + n;
                        if (p.mode == EPI_ACCUM_F32) {
                            v0 += o[0];
                            if (two) v1 += o[1];
                        } else if (p.mode == EPI_RESID_F32) {
                            const float* r = p.resid + (long)m * p.ldr + n;
                            v0 += r[0];
                            if (two) v1 += r[1];
                        }
                        o[0] = v0;
                        if (two) o[1] = v1;
                        break;
                    }
                    case EPI_ATOMIC_F32: {
                        float* o = static_cast<float*>(p.out) + (long)m * p.ldo + n;
                        atomicAdd(o, v0);
                        if (two) atomicAdd(o + 1, v1);
                        break;
                    }
                    case EPI_STORE_F16:
                    case EPI_BIAS_F16:
                    case EPI_GELU:
                    case EPI_GELU_D:
                    case EPI_GELU_BWD:
                    case EPI_GELU_BWD_D: {
                        if (p.mode == EPI_BIAS_F16) {
                            v0 += p.bias[n];
                            if (two) v1 += p.bias[n + 1];
                        } else if (p.mode == EPI_GELU) {
                            f16* a = p.aux + (long)m * p.ldaux + n;
                            // the backward differentiates at the stored (rounded) value
                            const f16 z0 = __float2half_rn(v0), z1 = __float2half_rn(v1);
                            a[0] = z0;
                            if (two) a[1] = z1;
                            v0 = gelu_as(__half2float(z0));
                            v1 = gelu_as(__half2float(z1));
                        } else if (p.mode == EPI_GELU_D) {
                            f16* a = p.aux + (long)m * p.ldaux + n;
                            float g0, d0, g1, d1;
                            gelu_as_pair(__half2float(__float2half_rn(v0)), g0, d0);
                            gelu_as_pair(__half2float(__float2half_rn(v1)), g1, d1);
                            a[0] = __float2half_rn(d0);
                            if (two) a[1] = __float2half_rn(d1);
                            v0 = g0;
                            v1 = g1;
                        } else if (p.mode == EPI_GELU_BWD || p.mode == EPI_GELU_BWD_D) {
                            const f16* z = p.auxin + (long)m * p.ldauxin + n;
                            if (p.mode == EPI_GELU_BWD) {
                                v0 *= gelu_as_grad(__half2float(z[0]));
                                if (two) v1 *= gelu_as_grad(__half2float(z[1]));
                            } else {
                                v0 *= __half2float(z[0]);
                                if (two) v1 *= __half2float(z[1]);
                            }
                            if (p.colscale2) {
                                v0 *= p.colscale2[n];
                                if (two) v1 *= p.colscale2[n + 1];
                            }
                        }
                        f16* o = static_cast<f16*>(p.out) + (long)m * p.ldo + n;
                        if (two && ((((long)m * p.ldo + n) & 1) == 0))
                            *reinterpret_cast<uint32_t*>(o) = pack_f16(v0, v1);
                        else {
                            o[0] = __float2half_rn(v0);
                            if (two) o[1] = __float2half_rn(v1);
                        }
                        break;
                    }
                }
            }
}

template <int BM, int BN, int WM_, int WN_, bool AK, bool BKM, int BK = 32, int STAGES = 4>
void launch(const GemmArgs& a, cudaStream_t s) {
    using S = Smem<BM, BN, AK, BKM, BK, STAGES>;
    auto kern = gemm_mma_kernel<BM, BN, WM_, WN_, AK, BKM, BK, STAGES>;
    static DeviceOnce once;  // per instantiation and device; before the first launch / capture
    once([&] { cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::BYTES); });
    dim3 grid((a.N + BN - 1) / BN, (a.M + BM - 1) / BM, a.splitk);
    launch_pdl(kern, grid, dim3(WM_ * WN_ * 32), S::BYTES, s, a);
}

template <bool AK, bool BKM>
void dispatch(const GemmArgs& a, cudaStream_t s) {
    // rank-block shapes are HBM-bound: small tiles (enough CTAs for every SM), deep pipelines
    if (a.N <= 32)                  // u = s X A^T, dU = s dY B (rows x 32); dB += dY^T U
        launch<64, 32, 4, 1, AK, BKM, 64, 6>(a, s);
    else if (a.M <= 32 && !AK)      // dA += dU^T X: 32 x in, split over rows
        launch<32, 128, 2, 4, AK, BKM, 64, 6>(a, s);
    else if (a.N <= 64)
        launch<128, 64, 4, 1, AK, BKM>(a, s);
    else if (a.M <= 64)
        launch<64, 128, 1, 4, AK, BKM>(a, s);
    else
        launch<128, 128, 2, 4, AK, BKM>(a, s);
}

}  // namespace

void gemm(const GemmArgs& a, cudaStream_t s) {
    if (a.M <= 0 || a.N <= 0 || (a.K1 <= 0 && a.K2 <= 0)) return;
    if ((a.a_kmajor || a.b_kmajor) && ((a.K1 % 8) || (a.K2 % 8)))
        throw std::runtime_error("gemm: K segments of a K-major operand must be multiples of 8");
    if ((!a.a_kmajor && (a.M % 8)) || (!a.b_kmajor && (a.N % 8)))
        throw std::runtime_error("gemm: MN-major operand extent must be a multiple of 8");
    if (a.a_kmajor) {
        if (a.b_kmajor) dispatch<true, true>(a, s);
        else dispatch<true, false>(a, s);
    } else {
        if (a.b_kmajor) dispatch<false, true>(a, s);
        else dispatch<false, false>(a, s);
    }
}

}  // namespace act
