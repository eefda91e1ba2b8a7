// elementwise.cu -- row / element kernels of the adapter training step (HBM-bound work).
#include <cuda_fp16.h>

#include <algorithm>
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"
#include "philox.cuh"

namespace act {

namespace {


// ---------------------------------------------------------------------------------------
// LayerNorm, src/ac/lora.h:86-93: mean, centre, x / sqrt(mean(x^2) + eps), * w + b.
template <int NV>
__global__ void ln_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                              const float* __restrict__ b, const float* __restrict__ add,
                              int rows_per_clip, f16* __restrict__ y, float* __restrict__ mean,
                              float* __restrict__ rstd, int rows, int D, float eps) {
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    constexpr int MAXV = NV;
    const int nv = NV;
    const float4* xr = reinterpret_cast<const float4*>(x + (long)row * D);
    float4 v[MAXV];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i)
        if (i < nv) {
            v[i] = xr[i * 32 + lane];
            s += v[i].x + v[i].y + v[i].z + v[i].w;
        }
    s = warp_sum(s);
    const float mu = s * (1.0f / (float)D);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i)
        if (i < nv) {
            const float a0 = v[i].x - mu, a1 = v[i].y - mu, a2 = v[i].z - mu, a3 = v[i].w - mu;
            ss += a0 * a0 + a1 * a1 + a2 * a2 + a3 * a3;
        }
    ss = warp_sum(ss);
    const float rs = 1.0f / sqrtf(ss / (float)D + eps);
    if (lane == 0) {
        mean[row] = mu;
        rstd[row] = rs;
    }
    const float* ad = add ? add + (long)(row / rows_per_clip) * D : nullptr;
#pragma unroll
    for (int i = 0; i < MAXV; ++i)
        if (i < nv) {
            const int j = (i * 32 + lane) * 4;
            const float4 ww = *reinterpret_cast<const float4*>(w + j);
            const float4 bb = *reinterpret_cast<const float4*>(b + j);
            float o0 = (v[i].x - mu) * rs * ww.x + bb.x, o1 = (v[i].y - mu) * rs * ww.y + bb.y;
            float o2 = (v[i].z - mu) * rs * ww.z + bb.z, o3 = (v[i].w - mu) * rs * ww.w + bb.w;
            if (ad) {
                const float4 aa = *reinterpret_cast<const float4*>(ad + j);
                o0 += aa.x; o1 += aa.y; o2 += aa.z; o3 += aa.w;
            }
            uint2 pk = make_uint2(pack_f16(o0, o1), pack_f16(o2, o3));
            *reinterpret_cast<uint2*>(y + (long)row * D + j) = pk;
        }
}

template <int NV>
__global__ void ln_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                              const float* __restrict__ w, const float* __restrict__ mean,
                              const float* __restrict__ rstd, float* __restrict__ dx, int accumulate,
                              const float* __restrict__ extra, f16* __restrict__ dx_h,
                              const float* __restrict__ colscale, int rows, int D) {
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    constexpr int MAXV = NV;
    const int nv = NV;
    const float mu = mean[row], rs = rstd[row];
    // every load of the row is issued before the reductions: dy, x, and the terms added to the
    // result (the accumulated dx and the extra gradient), so that their latencies overlap
    float4 gv[MAXV], xh[MAXV], ad[MAXV];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i)
        if (i < nv) {
            const int j = (i * 32 + lane) * 4;
            const float4 d = *reinterpret_cast<const float4*>(dy + (long)row * D + j);
            const float4 xx = *reinterpret_cast<const float4*>(x + (long)row * D + j);
            const float4 ww = *reinterpret_cast<const float4*>(w + j);
            ad[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (accumulate) ad[i] = *reinterpret_cast<const float4*>(dx + (long)row * D + j);
            if (extra) {
                const float4 e = *reinterpret_cast<const float4*>(extra + (long)row * D + j);
                ad[i].x += e.x; ad[i].y += e.y; ad[i].z += e.z; ad[i].w += e.w;
            }
            gv[i] = make_float4(d.x * ww.x, d.y * ww.y, d.z * ww.z, d.w * ww.w);
            xh[i] = make_float4((xx.x - mu) * rs, (xx.y - mu) * rs, (xx.z - mu) * rs, (xx.w - mu) * rs);
            s1 += gv[i].x + gv[i].y + gv[i].z + gv[i].w;
            s2 += gv[i].x * xh[i].x + gv[i].y * xh[i].y + gv[i].z * xh[i].z + gv[i].w * xh[i].w;
        }
    s1 = warp_sum(s1) / (float)D;
    s2 = warp_sum(s2) / (float)D;
#pragma unroll
    for (int i = 0; i < MAXV; ++i)
        if (i < nv) {
            const int j = (i * 32 + lane) * 4;
            float4* dp = reinterpret_cast<float4*>(dx + (long)row * D + j);
            float4 r = make_float4(rs * (gv[i].x - s1 - xh[i].x * s2), rs * (gv[i].y - s1 - xh[i].y * s2),
                                   rs * (gv[i].z - s1 - xh[i].z * s2), rs * (gv[i].w - s1 - xh[i].w * s2));
            r.x += ad[i].x; r.y += ad[i].y; r.z += ad[i].z; r.w += ad[i].w;
            *dp = r;
            if (dx_h) {
                float4 c = make_float4(1.f, 1.f, 1.f, 1.f);
                if (colscale) c = *reinterpret_cast<const float4*>(colscale + j);
                *reinterpret_cast<uint2*>(dx_h + (long)row * D + j) =
                    make_uint2(pack_f16(r.x * c.x, r.y * c.y), pack_f16(r.z * c.z, r.w * c.w));
            }
        }
}

__global__ void resid_f16_kernel(float* __restrict__ x, const float* __restrict__ extra,
                                  f16* __restrict__ dst, const float* __restrict__ colscale, long n4, int D) {
    pdl_wait();
    pdl_trigger();
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    float4 v = reinterpret_cast<float4*>(x)[i];
    if (extra) {
        const float4 e = reinterpret_cast<const float4*>(extra)[i];
        v.x += e.x; v.y += e.y; v.z += e.z; v.w += e.w;
        reinterpret_cast<float4*>(x)[i] = v;
    }
    float4 c = make_float4(1.f, 1.f, 1.f, 1.f);
    if (colscale) c = *reinterpret_cast<const float4*>(colscale + (i * 4) % D);
    reinterpret_cast<uint2*>(dst)[i] = make_uint2(pack_f16(v.x * c.x, v.y * c.y), pack_f16(v.z * c.z, v.w * c.w));
}

__global__ void f32_f16_kernel(const float* __restrict__ x, f16* __restrict__ y, long n) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __float2half_rn(x[i]);
}

// ---------------------------------------------------------------------------------------
// MelodyFlow inputs and loss, src/mf/train.h:154-159 and :107-108, src/mf/dit.h:172-173,208-216.
// An edit-bridge sample (start >= 0) replaces its noise with the t = 0 endpoint of the straight
// pivot -> clean bridge, (pivot - start*clean) / (1 - start) (src/mf/train.h:196-203), in the
// reference's float operations, each rounded once (no contraction into an FMA).
__global__ void mf_inputs_kernel(const float* __restrict__ clean, const float* __restrict__ noise,
                                 const float* __restrict__ tv, const float* __restrict__ start, int clips,
                                 int T, int lat, f16* __restrict__ x0, float* __restrict__ vstar) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const long n = (long)clips * lat * T;
    if (i >= n) return;
    const int b = (int)(i / ((long)lat * T));
    const int c = (int)((i / T) % lat), p = (int)(i % T);
    const float t = tv[b];
    const float rescale = 1.0f / sqrtf(t * t + (1.0f - t) * (1.0f - t));
    const float cl = clean[i], st = start[b];
    float nz = noise[i];
    if (st >= 0.0f) nz = __fdiv_rn(__fsub_rn(nz, __fmul_rn(st, cl)), __fsub_rn(1.0f, st));
    x0[((long)b * T + p) * lat + c] = __float2half_rn(((1 - t) * nz + t * cl) * rescale);
    vstar[i] = cl - nz;
}

// On-device posterior sampling: clean = mean + stddev * z and noise = z' with z, z' ~ N(0,1) by
// Box-Muller from one Philox4x32-10 call per two elements, keyed by `seed` and counted by
// (element pair, window): the draw of an element depends only on the seed, its window number and
// its index.  clean holds the mean and noise the stddev on entry (both [clips][lat * T]).
__global__ void mf_sample_kernel(float* __restrict__ clean, float* __restrict__ noise, int clips, long per_clip,
                                 uint64_t seed, uint64_t window0) {
    const long pairs = (per_clip + 1) / 2;
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)clips * pairs) return;
    const int b = (int)(i / pairs);
    const long p = i % pairs;
    const uint64_t w = window0 + (uint64_t)b;
    const Philox4 r = philox4x32_10((uint32_t)p, (uint32_t)w, (uint32_t)(w >> 32), 0x4D46u, (uint32_t)seed,
                                    (uint32_t)(seed >> 32));
    float z[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const float rad = sqrtf(-2.0f * logf(philox_open01(r.v[2 * h])));
        float sn, cs;
        sincospif(2.0f * philox_01(r.v[2 * h + 1]), &sn, &cs);
        z[2 * h] = rad * cs;
        z[2 * h + 1] = rad * sn;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const long e = 2 * p + h;
        if (e >= per_clip) break;
        const long at = (long)b * per_clip + e;
        const float m = clean[at], sd = noise[at];
        clean[at] = m + sd * z[2 * h];
        noise[at] = z[2 * h + 1];
    }
}

// MSE of the rescaled output against v* (flow target) and its seed gradient, multiplied by the
// backward's gradient scale gscale (a power of two; see kernels.h).  out / dout are
// [clips][T][lat] (token-major), vstar [clips][lat][T]; block (b, j) takes a strided share of
// clip b in out's order (coalesced out / dout) and leaves its partial sum in part[b][j].
constexpr int LOSS_PARTS = 32;
__global__ void mf_loss_part_kernel(const float* __restrict__ out, const float* __restrict__ vstar, int T,
                                    int lat, float* __restrict__ part, f16* __restrict__ dout, float gscale) {
    const int b = blockIdx.x, j = blockIdx.y;
    const long n = (long)T * lat;
    const float inv = 1.0f / (float)n, seed = 2.0f * sqrtf(2.0f) * inv * gscale;
    const float sq2 = sqrtf(2.0f);
    float acc = 0.f;
    for (long i = (long)j * blockDim.x + threadIdx.x; i < n; i += (long)LOSS_PARTS * blockDim.x) {
        const int p = (int)(i / lat), c = (int)(i % lat);
        const long o = (long)b * n + i;
        const float d = out[o] * sq2 - vstar[(long)b * n + (long)c * T + p];
        acc += d * d;
        dout[o] = __float2half_rn(d * seed);
    }
    __shared__ float red[32];
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) part[b * LOSS_PARTS + j] = v;
    }
}

// loss[b] = sum of clip b's partials / (T * lat), in a fixed order
__global__ void mf_loss_sum_kernel(const float* __restrict__ part, int clips, float inv, float* __restrict__ loss) {
    const int b = threadIdx.x;
    if (b >= clips) return;
    float v = 0.f;
    for (int j = 0; j < LOSS_PARTS; ++j) v += part[b * LOSS_PARTS + j];
    loss[b] = v * inv;
}

__global__ void linear_f32_kernel(const float* __restrict__ x, const float* __restrict__ W,
                                  float* __restrict__ y, int rows, int N, int K, int act) {
    const long w = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (w >= (long)rows * N) return;
    const int r = (int)(w / N), n = (int)(w % N);
    float acc = 0.f;
    for (int k = lane; k < K; k += 32) acc += x[(long)r * K + k] * W[(long)n * K + k];
    acc = warp_sum(acc);
    if (lane == 0) y[w] = act == 1 ? acc / (1.0f + expf(-acc)) : acc;
}

// ---------------------------------------------------------------------------------------
// DoRA-rows, src/ac/lora.h:62-79 (and the hand-derived backward of that factorisation).
// Column sums of a * b over the rows in at most DORA_COLSUM_PARTS row blocks.  A block takes 256
// columns (8 per lane, 16-byte loads) and one row block, its 8 warps taking every 8th row; the
// warps' sums meet in shared memory and are added in warp order, and the block leaves its
// partial in part[row block][n].  The last block of a column block to finish (a counter per
// column block, reset by that block) adds the row blocks' partials in row-block order, so the
// sum does not depend on the order in which blocks finish, and applies the DoRA factor.
__global__ void __launch_bounds__(256) dora_colsum_kernel(const f16* __restrict__ a, long lda,
                                                          const f16* __restrict__ b, long ldb, int rows, int N,
                                                          float* __restrict__ part, int rows_per_block,
                                                          int* __restrict__ count, const float* __restrict__ g,
                                                          float* __restrict__ dg, float inv_gscale) {
    __shared__ float red[8][256];
    __shared__ int last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c0 = blockIdx.x * 256 + lane * 8;
    const int r0 = blockIdx.y * rows_per_block, r1 = min(rows, r0 + rows_per_block);
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    if (c0 < N) {
        for (int r = r0 + warp; r < r1; r += 8) {
            const uint4 x = *reinterpret_cast<const uint4*>(a + (long)r * lda + c0);
            const uint4 y = *reinterpret_cast<const uint4*>(b + (long)r * ldb + c0);
            const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 u = unpack_f16(xs[e]), v = unpack_f16(ys[e]);
                acc[2 * e] += u.x * v.x;
                acc[2 * e + 1] += u.y * v.y;
            }
        }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) red[warp][lane * 8 + e] = acc[e];
    __syncthreads();
    const int n = blockIdx.x * 256 + threadIdx.x;
    if (n < N) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) v += red[w][threadIdx.x];
        part[(long)blockIdx.y * N + n] = v;
    }
    __threadfence();  // this block's partial is visible before it is counted
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(count + blockIdx.x, 1) == (int)gridDim.y - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (n < N) {
        float t = 0.f;
#pragma unroll 8
        for (int j = 0; j < (int)gridDim.y; ++j) t += __ldcg(part + (long)j * N + n);  // row-block order
        const float gg = g[n];
        dg[n] += t * inv_gscale / (gg * gg);
    }
    if (threadIdx.x == 0) count[blockIdx.x] = 0;  // ready for the next launch
}

// The per-step factors and the backward tail are batched: one launch covers a list of
// projections (blockIdx.y), so the whole model's factors, or one layer's tails, cost one launch
// per stage instead of one per projection.  Blocks past a projection's own size exit.

// sum of one value per thread over a block of 256 threads, in a fixed order; thread 0 has it
__device__ __forceinline__ float block_sum256(float acc) {
    __shared__ float red[8];
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    float v = 0.f;
    if (threadIdx.x < 32) {
        v = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
        v = warp_sum(v);
    }
    return v;
}

// G = A A^T [r][r], one block per entry
__global__ void __launch_bounds__(256) dora_gram_a_kernel(const DoraJob* __restrict__ jobs) {
    const DoraJob J = jobs[blockIdx.y];
    if ((int)blockIdx.x >= J.r * J.r) return;
    const int j = blockIdx.x / J.r, k = blockIdx.x % J.r;
    float acc = 0.f;
    for (int i = threadIdx.x; i < J.in; i += 256) acc += J.A[(long)j * J.in + i] * J.A[(long)k * J.in + i];
    acc = block_sum256(acc);
    if (threadIdx.x == 0) J.G[blockIdx.x] = acc;
}

// One warp per output row: Q[o] = B[o] G, nsq = ||W_o||^2 + in*1e-12 + 2s<W_o,(BA)_o> + s^2 B[o]·Q[o]
// (P[o] = (W A^T)[o] gives <W_o,(BA)_o> = P[o]·B[o]), g = m / sqrt(nsq); lanes take the rank
// columns, then a fixed-order warp sum.  The row's column-sum accumulator dg starts at zero.
__global__ void __launch_bounds__(256) dora_rows_kernel(const DoraJob* __restrict__ jobs) {
    const DoraJob J = jobs[blockIdx.y];
    const int o = blockIdx.x * 8 + threadIdx.x / 32, lane = threadIdx.x & 31;
    if (o >= J.out) return;
    const int r = J.r;
    const float* b = J.B + (long)o * r;
    float t2 = 0.f, t3 = 0.f;
    for (int j = lane; j < r; j += 32) {
        float qv = 0.f;
        for (int k = 0; k < r; ++k) qv += b[k] * J.G[k * r + j];
        J.Q[(long)o * r + j] = qv;
        t2 += J.P[(long)o * J.RP + j] * b[j];
        t3 += b[j] * qv;
    }
    t2 = warp_sum(t2);
    t3 = warp_sum(t3);
    if (lane == 0) {
        const float n = J.base[o] + 2.0f * J.s * t2 + J.s * J.s * t3;
        J.nsq[o] = n;
        J.g[o] = J.m[o] / sqrtf(n);
        J.dg[o] = 0.f;
    }
}

// One warp per output row: gm += dg / sqrt(nsq); dt2 = 2s dnsq, dt3 = s^2 dnsq (kept in scr);
// gB[o] += dt2 P[o] + 2 dt3 Q[o] and BD[o] = f16(bd_scale dt2 B[o]) (zero past r), lanes along
// the rank columns so every row's loads and stores are contiguous.
__global__ void __launch_bounds__(256) dora_tail_kernel(const DoraJob* __restrict__ jobs, float bd_scale) {
    const DoraJob J = jobs[blockIdx.y];
    const int o = blockIdx.x * 8 + threadIdx.x / 32, lane = threadIdx.x & 31;
    if (o >= J.out) return;
    const float dg = J.dg[o], nsq = J.nsq[o];
    const float sq = sqrtf(nsq);
    const float dn = -0.5f * dg * J.g[o] / nsq;
    const float d2 = 2.0f * J.s * dn, d3 = J.s * J.s * dn;
    if (lane == 0) {
        J.gm[o] += dg / sq;
        J.scr[o] = d3;
    }
    for (int j = lane; j < J.RP; j += 32) {
        if (j < J.r) {
            J.gB[(long)o * J.r + j] += d2 * J.P[(long)o * J.RP + j] + 2.0f * d3 * J.Q[(long)o * J.r + j];
            J.BD[(long)o * J.RP + j] = __float2half_rn(bd_scale * d2 * J.B[(long)o * J.r + j]);
        } else {
            J.BD[(long)o * J.RP + j] = __float2half_rn(0.f);
        }
    }
}

// dG = B^T diag(dt3) B [r][r] into scr + out, one block per entry
__global__ void __launch_bounds__(256) dora_gram_b_kernel(const DoraJob* __restrict__ jobs) {
    const DoraJob J = jobs[blockIdx.y];
    if ((int)blockIdx.x >= J.r * J.r) return;
    const int r = J.r, j = blockIdx.x / r, k = blockIdx.x % r;
    float acc = 0.f;
    for (int o = threadIdx.x; o < J.out; o += 256) acc += J.scr[o] * J.B[(long)o * r + j] * J.B[(long)o * r + k];
    acc = block_sum256(acc);
    if (threadIdx.x == 0) J.scr[J.out + blockIdx.x] = acc;
}

// gA [r][in] += 2 dG A
__global__ void __launch_bounds__(256) dora_ga_kernel(const DoraJob* __restrict__ jobs) {
    const DoraJob J = jobs[blockIdx.y];
    const long e = (long)blockIdx.x * 256 + threadIdx.x;
    if (e >= (long)J.r * J.in) return;
    const int r = J.r, j = (int)(e / J.in), i = (int)(e % J.in);
    const float* dG = J.scr + J.out;
    float acc = 0.f;
    for (int k = 0; k < r; ++k) acc += dG[j * r + k] * J.A[(long)k * J.in + i];
    J.gA[e] += 2.0f * acc;
}

// ---------------------------------------------------------------------------------------
__global__ void refresh_kernel(const CopyJob* jobs) {
    const CopyJob j = jobs[blockIdx.y];
    const long n = (long)j.rows * j.cols;
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long)gridDim.x * blockDim.x) {
        const int row = (int)(e / j.cols), col = (int)(e % j.cols);
        j.dst[(long)row * j.ldd + col] = __float2half_rn(j.src[e]);
    }
}

// ---------------------------------------------------------------------------------------
// AdamW, src/ac/train_controls.h:89-118: mean over microbatches, global-norm clip, decoupled
// decay on lora_A / lora_B only.
__global__ void grad_norm_kernel(const float* __restrict__ grad, long n, float count,
                                 double* __restrict__ partials) {
    double acc = 0.0;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const float x = grad[i] / count;
        acc += (double)x * x;
    }
    __shared__ double red[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        double v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) partials[blockIdx.x] = v;
    }
}

__global__ void adamw_kernel(float* __restrict__ value, float* __restrict__ m, float* __restrict__ v,
                             float* __restrict__ grad, const uint8_t* __restrict__ decay_mask, long n,
                             float count, float clip, float lr, float beta1, float beta2, float eps,
                             float decay, float bc1, float bc2, const double* __restrict__ partials,
                             int nparts, int* __restrict__ nonfinite) {
    __shared__ float sscale;
    if (threadIdx.x < 32) {
        double acc = 0.0;
        for (int i = threadIdx.x; i < nparts; i += 32) acc += partials[i];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (threadIdx.x == 0) sscale = (float)fmin(1.0, (double)clip / (sqrt(acc) + 1e-12));
    }
    __syncthreads();
    const float scale = sscale;
    int bad = 0;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const float wd = decay_mask[i] ? decay : 0.0f;
        const float gr = scale * (grad[i] / count);
        const float mi = beta1 * m[i] + (1 - beta1) * gr;
        const float vi = beta2 * v[i] + (1 - beta2) * gr * gr;
        const float val = value[i] - lr * ((mi / bc1) / (sqrtf(vi / bc2) + eps) + wd * value[i]);
        m[i] = mi;
        v[i] = vi;
        value[i] = val;
        grad[i] = 0.f;
        bad += !isfinite(val);
    }
    if (bad) atomicAdd(nonfinite, bad);
}

// ---------------------------------------------------------------------------------------
// Q8_0: 34-byte blocks {fp16 d; int8 q[32]}; w = d * q exactly in fp32 (then rounded to the
// f16 GEMM operand).
__global__ void q8_f16_kernel(const uint8_t* __restrict__ blocks, long nblocks, f16* __restrict__ out) {
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= nblocks * 32) return;
    const uint8_t* blk = blocks + (e >> 5) * 34;
    const __half d = __ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8)));
    out[e] = __float2half_rn(__half2float(d) * (float)(int8_t)blk[2 + (e & 31)]);
}

// Q8_0 weight [rows][cols] split into its quants biased to unsigned ([rows][cols], q + 128) and
// its scales transposed ([cols / 32][rows]); one block per thread.
__global__ void q8_split_kernel(const uint8_t* __restrict__ blocks, int rows, int cols, uint8_t* __restrict__ q,
                                f16* __restrict__ d) {
    const long b = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const int nb = cols / 32;
    if (b >= (long)rows * nb) return;
    const int r = (int)(b / nb), j = (int)(b % nb);
    const uint8_t* blk = blocks + b * 34;
    d[(long)j * rows + r] = __ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8)));
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
        w[i] = (blk[2 + 4 * i] | (blk[3 + 4 * i] << 8) | (blk[4 + 4 * i] << 16) | ((uint32_t)blk[5 + 4 * i] << 24)) ^
               0x80808080u;
    uint4* dst = reinterpret_cast<uint4*>(q + (long)r * cols + j * 32);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

// A Q8_0 weight view as f16 (biased quants, transposed scales); 8 columns per thread.
__global__ void q8_view_f16_kernel(const uint8_t* __restrict__ q, long ldq, const f16* __restrict__ d, long ldd,
                                   int rows, int cols, f16* __restrict__ out, long ldo) {
    const long e = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (e >= (long)rows * cols) return;
    const int r = (int)(e / cols), c = (int)(e % cols);
    const float sc = __half2float(d[(long)(c / 32) * ldd + r]);
    const uint8_t* qr = q + (long)r * ldq + c;
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
        o[j] = pack_f16(sc * (float)((int)qr[2 * j] - 128), sc * (float)((int)qr[2 * j + 1] - 128));
    *reinterpret_cast<uint4*>(out + (long)r * ldo + c) = make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void q8_f32_kernel(const uint8_t* __restrict__ blocks, long nblocks, float* __restrict__ out) {
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= nblocks * 32) return;
    const uint8_t* blk = blocks + (e >> 5) * 34;
    const __half d = __ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8)));
    out[e] = __half2float(d) * (float)(int8_t)blk[2 + (e & 31)];
}

// ---------------------------------------------------------------------------------------
// MusicGen: summed codebook embeddings plus sinusoidal positions (src/mg/train.h:17-22).
__global__ void mg_embed_kernel(const int32_t* __restrict__ ids, int steps, int nq,
                                const float* const* __restrict__ emb, const float* __restrict__ pos,
                                float* __restrict__ x, int D, int seqs) {
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (long)seqs * steps * D) return;
    const int j = (int)(e % D);
    const long row = e / D;
    const int b = (int)(row / steps), s = (int)(row % steps);
    float acc = 0.f;
    for (int q = 0; q < nq; ++q) {
        const int id = ids[((long)b * nq + q) * steps + s];
        acc += emb[q][(long)id * D + j];
    }
    x[e] = acc + pos[(long)s * D + j];
}

// ggml_cross_entropy_loss over the selected rows, src/mg/train.h:131.
// Each row leaves its loss term in rowloss[row]; mg_loss_add_kernel sums them in row order.
__global__ void mg_ce_kernel(const float* __restrict__ logits, int sel, int T, int row0, int card,
                             const int32_t* __restrict__ targets, long tgt_stride, float inv_nsel,
                             float* __restrict__ rowloss, f16* __restrict__ dlogits, float gscale) {
    const int row = blockIdx.x;  // scored row of the codebook, sample-major
    const int b = row / sel, st = row % sel;
    const int tgt = targets[(long)b * tgt_stride + st];
    const long lrow = (long)b * T + row0 + st;
    const float* lg = logits + lrow * card;
    f16* dl = dlogits + lrow * card;
    __shared__ float red[32];
    __shared__ float sh_max, sh_sum;
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < card; j += blockDim.x) mx = fmaxf(mx, lg[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (threadIdx.x == 0) sh_max = v;
    }
    __syncthreads();
    mx = sh_max;
    float sm = 0.f;
    for (int j = threadIdx.x; j < card; j += blockDim.x) sm += expf(lg[j] - mx);
    sm = warp_sum(sm);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sm;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) sh_sum = v;
    }
    __syncthreads();
    sm = sh_sum;
    if (tgt < 0) {
        for (int j = threadIdx.x; j < card; j += blockDim.x) dl[j] = __float2half_rn(0.f);
        if (threadIdx.x == 0) rowloss[row] = 0.f;
        return;
    }
    const float inv = 1.0f / sm, seed = inv_nsel * gscale;
    for (int j = threadIdx.x; j < card; j += blockDim.x)
        dl[j] = __float2half_rn((expf(lg[j] - mx) * inv - (j == tgt ? 1.0f : 0.0f)) * seed);
    if (threadIdx.x == 0) rowloss[row] = (mx + logf(sm) - lg[tgt]) * inv_nsel;
}

// loss_acc[seq] += the row terms of seq in a fixed order (one block per sequence): the printed
// loss does not depend on the order in which rows finished
__global__ void mg_loss_add_kernel(const float* __restrict__ rowloss, int rows, int rows_per_seq,
                                   float* __restrict__ loss_acc) {
    const int seq = blockIdx.x;
    const int r0 = seq * rows_per_seq, r1 = min(rows, r0 + rows_per_seq);
    float v = 0.f;
    for (int r = r0 + (int)threadIdx.x; r < r1; r += blockDim.x) v += rowloss[r];
    __shared__ float red[32];
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        float w = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
        w = warp_sum(w);
        if (threadIdx.x == 0) loss_acc[seq] += w;
    }
}

// gact = gelu(z); with store_grad, z is overwritten by gelu'(z).  8 f16 per thread and step;
// the A&S evaluation of gelu_as_pair on each f16 pre-activation (the pass stays HBM-bound).
__global__ void __launch_bounds__(256) gelu_fwd_kernel(f16* __restrict__ z, f16* __restrict__ gact, long n8,
                                                       int store_grad) {
    pdl_wait();
    pdl_trigger();
    for (long c = (long)blockIdx.x * blockDim.x + threadIdx.x; c < n8; c += (long)gridDim.x * blockDim.x) {
        const uint4 zz = reinterpret_cast<const uint4*>(z)[c];
        const uint32_t w[4] = {zz.x, zz.y, zz.z, zz.w};
        uint32_t g[4], d[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 x = unpack_f16(w[j]);
            float g0, d0, g1, d1;
            gelu_as_pair(x.x, g0, d0);
            gelu_as_pair(x.y, g1, d1);
            g[j] = pack_f16(g0, g1);
            d[j] = pack_f16(d0, d1);
        }
        reinterpret_cast<uint4*>(gact)[c] = make_uint4(g[0], g[1], g[2], g[3]);
        if (store_grad) reinterpret_cast<uint4*>(z)[c] = make_uint4(d[0], d[1], d[2], d[3]);
    }
}

// stand-alone check: gelu / gelu' of f16 inputs through the training step's pass
__global__ void gelu_check_kernel(const uint16_t* z, uint16_t* g, uint16_t* dg, long n) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float gv, dv;
    gelu_as_pair(__half2float(__ushort_as_half(z[i])), gv, dv);
    g[i] = __half_as_ushort(__float2half_rn(gv));
    dg[i] = __half_as_ushort(__float2half_rn(dv));
}

inline unsigned blocks_for(long n, int t) { return (unsigned)((n + t - 1) / t); }

}  // namespace

#define LN_DISPATCH(KERNEL, ...)                                                                  \
    switch (D / 128) {                                                                            \
        case 1: launch_pdl(KERNEL<1>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 2: launch_pdl(KERNEL<2>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 3: launch_pdl(KERNEL<3>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 4: launch_pdl(KERNEL<4>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 5: launch_pdl(KERNEL<5>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 6: launch_pdl(KERNEL<6>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 7: launch_pdl(KERNEL<7>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 8: launch_pdl(KERNEL<8>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 9: launch_pdl(KERNEL<9>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 10: launch_pdl(KERNEL<10>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 11: launch_pdl(KERNEL<11>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 12: launch_pdl(KERNEL<12>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 13: launch_pdl(KERNEL<13>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 14: launch_pdl(KERNEL<14>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 15: launch_pdl(KERNEL<15>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        case 16: launch_pdl(KERNEL<16>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, __VA_ARGS__); break; \
        default: break; /* rejected at context creation: D must be 128..2048, a multiple of 128 */ \
    }

void layernorm_fwd(const float* x, const float* w, const float* b, const float* add, int rows_per_clip,
                   f16* y, float* mean, float* rstd, int rows, int D, float eps, cudaStream_t s) {
    LN_DISPATCH(ln_fwd_kernel, x, w, b, add, rows_per_clip, y, mean, rstd, rows, D, eps);
}

void layernorm_bwd(const float* dy, const float* x, const float* w, const float* mean, const float* rstd,
                   float* dx, int accumulate, const float* extra, f16* dx_h, const float* colscale,
                   int rows, int D, cudaStream_t s) {
    LN_DISPATCH(ln_bwd_kernel, dy, x, w, mean, rstd, dx, accumulate, extra, dx_h, colscale, rows, D);
}

void residual_to_f16(float* x, const float* extra, f16* dst, const float* colscale, int rows, int D,
                      cudaStream_t s) {
    const long n4 = (long)rows * D / 4;
    launch_pdl(resid_f16_kernel, dim3(blocks_for(n4, 256)), dim3(256), 0, s, x, extra, dst, colscale, n4, D);
}

void gelu_check(const uint16_t* z, uint16_t* g, uint16_t* dg, long n, cudaStream_t s) {
    gelu_check_kernel<<<blocks_for(n, 256), 256, 0, s>>>(z, g, dg, n);
}

void gelu_fwd(f16* z, f16* gact, long n, int store_grad, cudaStream_t s) {
    const long n8 = n / 8;
    long blocks = std::min<long>(blocks_for(n8, 256), 148L * 8);
    launch_pdl(gelu_fwd_kernel, dim3((unsigned)blocks), dim3(256), 0, s, z, gact, n8, store_grad);
}

void f32_to_f16(const float* x, f16* y, long n, cudaStream_t s) {
    f32_f16_kernel<<<blocks_for(n, 256), 256, 0, s>>>(x, y, n);
}

void mf_sample(float* clean, float* noise, int clips, long per_clip, uint64_t seed, uint64_t window0, cudaStream_t s) {
    const long n = (long)clips * ((per_clip + 1) / 2);
    mf_sample_kernel<<<blocks_for(n, 256), 256, 0, s>>>(clean, noise, clips, per_clip, seed, window0);
}

void mf_inputs(const float* clean, const float* noise, const float* t, const float* start, int clips, int T,
               int lat, f16* x0, float* vstar, cudaStream_t s) {
    const long n = (long)clips * lat * T;
    mf_inputs_kernel<<<blocks_for(n, 256), 256, 0, s>>>(clean, noise, t, start, clips, T, lat, x0, vstar);
}

void mf_loss(const float* out, const float* vstar, int clips, int T, int lat, float* loss, f16* dout,
             float* part, float gscale, cudaStream_t s) {
    mf_loss_part_kernel<<<dim3(clips, LOSS_PARTS), 256, 0, s>>>(out, vstar, T, lat, part, dout, gscale);
    mf_loss_sum_kernel<<<1, 32 * ((clips + 31) / 32), 0, s>>>(part, clips, 1.0f / ((float)T * lat), loss);
}

void linear_f32(const float* x, const float* W, float* y, int rows, int N, int K, int act, cudaStream_t s) {
    linear_f32_kernel<<<blocks_for((long)rows * N, 8), 256, 0, s>>>(x, W, y, rows, N, K, act);
}

void dora_colsum(const f16* a, long lda, const f16* b, long ldb, int rows, int N, const float* colscale,
                 float* dg, float* part, int* count, float inv_gscale, cudaStream_t s) {
    if (N % 8 || lda % 8 || ldb % 8) throw std::runtime_error("dora_colsum: rows must be whole 16-byte pieces");
    // about four blocks per SM in all (the loads of a block are few and serial), each block at
    // least 64 rows: a fixed split for a given shape and device
    const int col_blocks = blocks_for(N, 256);
    const int want = std::max(1, (4 * current_sm_count() + col_blocks - 1) / col_blocks);
    const int nparts = std::min(std::min(want, DORA_COLSUM_PARTS), std::max(1, rows / 64));
    const int rpb = (rows + nparts - 1) / nparts;
    const int parts = (rows + rpb - 1) / rpb;
    dim3 grid(col_blocks, parts);
    dora_colsum_kernel<<<grid, 256, 0, s>>>(a, lda, b, ldb, rows, N, part, rpb, count, colscale, dg, inv_gscale);
}

void dora_factors(const DoraJob* jobs, int n, int r, int max_out, cudaStream_t st) {
    if (n <= 0) return;
    dora_gram_a_kernel<<<dim3(r * r, n), 256, 0, st>>>(jobs);
    dora_rows_kernel<<<dim3(blocks_for(max_out, 8), n), 256, 0, st>>>(jobs);
}

void dora_tail(const DoraJob* jobs, int n, int r, int max_out, int max_in, float bd_scale, cudaStream_t st) {
    if (n <= 0) return;
    dora_tail_kernel<<<dim3(blocks_for(max_out, 8), n), 256, 0, st>>>(jobs, bd_scale);
    dora_gram_b_kernel<<<dim3(r * r, n), 256, 0, st>>>(jobs);
    dora_ga_kernel<<<dim3(blocks_for((long)r * max_in, 256), n), 256, 0, st>>>(jobs);
}

void refresh_f16(const CopyJob* jobs_dev, int njobs, int max_elems, cudaStream_t s) {
    if (njobs <= 0) return;
    dim3 grid(blocks_for(max_elems, 256) > 256 ? 256 : blocks_for(max_elems, 256), njobs);
    refresh_kernel<<<grid, 256, 0, s>>>(jobs_dev);
}

void adamw(float* value, float* m, float* v, float* grad, const uint8_t* decay_mask, long n, float count,
           float clip, float lr, float beta1, float beta2, float eps, float decay, float bc1, float bc2,
           double* partials, int* nonfinite, cudaStream_t s) {
    const int nparts = 592;
    grad_norm_kernel<<<nparts, 256, 0, s>>>(grad, n, count, partials);
    adamw_kernel<<<592, 256, 0, s>>>(value, m, v, grad, decay_mask, n, count, clip, lr, beta1, beta2, eps,
                                     decay, bc1, bc2, partials, nparts, nonfinite);
}

void q8_0_to_f16(const uint8_t* blocks, long nblocks, f16* out, cudaStream_t s) {
    q8_f16_kernel<<<blocks_for(nblocks * 32, 256), 256, 0, s>>>(blocks, nblocks, out);
}

void q8_0_split(const uint8_t* blocks, int rows, int cols, uint8_t* q, f16* d, cudaStream_t s) {
    const long n = (long)rows * (cols / 32);
    q8_split_kernel<<<blocks_for(n, 256), 256, 0, s>>>(blocks, rows, cols, q, d);
}

void q8_view_to_f16(const uint8_t* q, long ldq, const f16* d, long ldd, int rows, int cols, f16* out, long ldo,
                    cudaStream_t s) {
    const long n8 = (long)rows * cols / 8;  // cols is a multiple of 32
    q8_view_f16_kernel<<<blocks_for(n8, 256), 256, 0, s>>>(q, ldq, d, ldd, rows, cols, out, ldo);
}

void q8_0_to_f32(const uint8_t* blocks, long nblocks, float* out, cudaStream_t s) {
    q8_f32_kernel<<<blocks_for(nblocks * 32, 256), 256, 0, s>>>(blocks, nblocks, out);
}

void mg_embed(const int32_t* ids, int steps, int nq, const float* const* emb_dev, const float* pos, float* x,
              int D, int seqs, cudaStream_t s) {
    const long n = (long)seqs * steps * D;
    mg_embed_kernel<<<blocks_for(n, 256), 256, 0, s>>>(ids, steps, nq, emb_dev, pos, x, D, seqs);
}

void mg_cross_entropy(const float* logits, int n, int sel, int T, int row0, int card, const int32_t* targets,
                      long tgt_stride, float inv_nsel, float* loss_acc, float* rowloss, f16* dlogits, float gscale,
                      cudaStream_t s) {
    if (n <= 0 || sel <= 0) return;
    mg_ce_kernel<<<n * sel, 256, 0, s>>>(logits, sel, T, row0, card, targets, tgt_stride, inv_nsel, rowloss, dlogits,
                                         gscale);
    mg_loss_add_kernel<<<n, 256, 0, s>>>(rowloss, n * sel, sel, loss_acc);
}

}  // namespace act
