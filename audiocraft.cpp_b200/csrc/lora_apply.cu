// lora_apply.cu -- adapter consumption at inference: lora_linear (src/ac/lora.h:50-83) on the
// device, for a caller that applies a trained adapter to a frozen projection (mf-edit --lora,
// mg generation with an adapter: tools/mf-edit.cpp:268-299).
//
//   base  = W x                              (the dense GEMM; Q8_0 weights dequantised inside it)
//   LoRA  : y = base + (strength * alpha / rank) * B (A x)
//   DoRA  : y_lin = base + s * B (A x),  s = alpha / rank
//           nsq_o = ||W_o||^2 + in * 1e-12 + 2 s <W_o, (BA)_o> + s^2 ||(BA)_o||^2
//           y = y_lin * m / sqrt(nsq);  strength != 1: y = base + strength * (y - base)
// ||W_o||^2 is accumulated in double on the host (lora_row_norm_sq, src/ac/lora.h:11-32); the
// rank-sized products run in fp32 on the device.
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "actrain.h"
#include "common.cuh"
#include "kernels.h"

namespace act {

namespace {

// nsq and the DoRA factor per output row: P = W A^T [out][r], G = A A^T [r][r]
__global__ void lora_dora_factor_kernel(const float* __restrict__ B, const float* __restrict__ P,
                                        const float* __restrict__ G, const float* __restrict__ base_nsq,
                                        const float* __restrict__ m, int out, int r, float s,
                                        float* __restrict__ g) {
    const int o = blockIdx.x * blockDim.x + threadIdx.x;
    if (o >= out) return;
    const float* b = B + (long)o * r;
    float t2 = 0.f, t3 = 0.f;
    for (int j = 0; j < r; ++j) {
        t2 += b[j] * P[(long)o * r + j];
        float gb = 0.f;
        for (int k = 0; k < r; ++k) gb += G[j * r + k] * b[k];
        t3 += b[j] * gb;
    }
    const float nsq = (base_nsq[o] + (2.0f * s) * t2) + (s * s) * t3;
    g[o] = m[o] / sqrtf(nsq);
}

// y = base + s * yd (LoRA), or the DoRA combination with strength blending
__global__ void lora_combine_kernel(float* __restrict__ y, const float* __restrict__ yd, long n, int out,
                                    float s, const float* __restrict__ g, float strength) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float base = y[i];
    float v = base + s * yd[i];
    if (g) {
        v = v * g[i % out];
        if (strength != 1.0f) v = base + (v - base) * strength;
    }
    y[i] = v;
}

}  // namespace

namespace {
float half_bits_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    int exp = (h >> 10) & 31;
    uint32_t man = h & 1023;
    uint32_t bits;
    if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else if (exp == 0) {
        if (!man) {
            bits = sign;
        } else {  // subnormal: normalise
            int e = -1;
            do {
                man <<= 1;
                ++e;
            } while (!(man & 1024));
            bits = sign | (uint32_t)(127 - 15 - e) << 23 | (man & 1023) << 13;
        }
    } else {
        bits = sign | (uint32_t)(exp - 15 + 127) << 23 | man << 13;
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// The weight's values as fp32 on the host (F32, F16 or Q8_0: d * q in fp32)
std::vector<float> host_weight(int type, const void* w, size_t bytes, long n) {
    std::vector<float> v((size_t)n);
    if (type == ACT_TYPE_F32) {
        if (bytes != (size_t)n * 4) throw std::invalid_argument("weight size mismatch");
        std::memcpy(v.data(), w, bytes);
    } else if (type == ACT_TYPE_F16) {
        if (bytes != (size_t)n * 2) throw std::invalid_argument("weight size mismatch");
        const uint16_t* h = static_cast<const uint16_t*>(w);
        for (long i = 0; i < n; ++i) v[(size_t)i] = half_bits_to_float(h[i]);
    } else if (type == ACT_TYPE_Q8_0) {
        if (n % 32 || bytes != (size_t)(n / 32) * 34) throw std::invalid_argument("weight size mismatch");
        const uint8_t* b = static_cast<const uint8_t*>(w);
        for (long k = 0; k < n / 32; ++k) {
            uint16_t dh;
            std::memcpy(&dh, b + 34 * k, 2);
            const float d = half_bits_to_float(dh);
            for (int j = 0; j < 32; ++j) v[(size_t)(32 * k + j)] = d * (float)(int8_t)b[34 * k + 2 + j];
        }
    } else {
        throw std::invalid_argument("unsupported weight type");
    }
    return v;
}

#define LCK(x)                                                                                   \
    do {                                                                                         \
        cudaError_t e_ = (x);                                                                    \
        if (e_ != cudaSuccess) throw std::runtime_error(std::string(#x) + ": " + cudaGetErrorString(e_)); \
    } while (0)

}  // namespace

// Throws std::invalid_argument for bad arguments and std::runtime_error for CUDA failures (the
// C ABI wrapper, act_lora_linear, maps them to status codes).
void lora_linear(int device, const float* x, int64_t rows, int in, int out, int w_type, const void* w,
                 size_t w_bytes, const float* A, const float* B, int rank, float alpha, const float* magnitude,
                 float strength, float* y) {
    std::vector<void*> bufs;
    cudaStream_t st = nullptr;
    auto cleanup = [&] {
        if (st) cudaStreamSynchronize(st);
        for (void* b : bufs) cudaFree(b);
        if (st) cudaStreamDestroy(st);
    };
    try {
        if (!x || !w || !y || rows <= 0 || in <= 0 || out <= 0 || (in % 8) || (out % 8))
            throw std::invalid_argument("invalid lora_linear arguments (in and out must be multiples of 8)");
        const bool adapted = A != nullptr;
        const bool dora = adapted && magnitude != nullptr;
        if (adapted && (!B || rank <= 0 || rank > 64 || !std::isfinite(alpha) || alpha <= 0 || !std::isfinite(strength)))
            throw std::invalid_argument("invalid adapter rank, alpha or strength");
        const long nw = (long)out * in;
        const std::vector<float> wh = (dora || w_type == ACT_TYPE_F32) ? host_weight(w_type, w, w_bytes, nw)
                                                                       : std::vector<float>();
        if (w_type != ACT_TYPE_F32 && w_type != ACT_TYPE_F16 && w_type != ACT_TYPE_Q8_0)
            throw std::invalid_argument("unsupported weight type");
        LCK(cudaSetDevice(device));
        LCK(cudaStreamCreate(&st));
        auto dev = [&](size_t bytes) -> void* {
            void* d = nullptr;
            LCK(cudaMalloc(&d, bytes < 16 ? 16 : bytes));
            bufs.push_back(d);
            return d;
        };
        auto up = [&](const void* h, size_t bytes) -> void* {
            void* d = dev(bytes);
            LCK(cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, st));
            return d;
        };
        int* derr = static_cast<int*>(dev(sizeof(int)));
        LCK(cudaMemsetAsync(derr, 0, sizeof(int), st));
        float* xd = static_cast<float*>(up(x, (size_t)rows * in * 4));
        f16* xh = static_cast<f16*>(dev((size_t)rows * in * 2));
        f32_to_f16(xd, xh, rows * in, st);
        float* yd = static_cast<float*>(dev((size_t)rows * out * 4));
        // base = W x on the tensor cores: f16 operands, fp32 accumulation
        GemmArgs g;
        g.M = (int)rows; g.N = out; g.K1 = in;
        g.A1 = xh; g.lda1 = in; g.b_kmajor = true;
        g.mode = EPI_STORE_F32; g.out = yd; g.ldo = out;
        if (w_type == ACT_TYPE_Q8_0) {
            if (w_bytes != (size_t)(nw / 32) * 34 || in % 32) throw std::invalid_argument("weight size mismatch");
            const uint8_t* blocks = static_cast<const uint8_t*>(up(w, w_bytes));
            uint8_t* q = static_cast<uint8_t*>(dev((size_t)nw));
            f16* dsc = static_cast<f16*>(dev((size_t)nw / 32 * 2));
            q8_0_split(blocks, out, in, q, dsc, st);
            g.B1q = q; g.ldb1 = in; g.B1d = dsc; g.ldd1 = out;
            if (!gemm_tc_supported(g)) {  // too few rows for the 2-CTA kernel: expand to f16 instead
                f16* wf = static_cast<f16*>(dev((size_t)nw * 2));
                q8_view_to_f16(q, in, dsc, out, out, in, wf, in, st);
                g.B1q = nullptr; g.B1d = nullptr; g.B1 = wf;
            }
        } else if (w_type == ACT_TYPE_F16) {
            if (w_bytes != (size_t)nw * 2) throw std::invalid_argument("weight size mismatch");
            g.B1 = static_cast<const f16*>(up(w, w_bytes)); g.ldb1 = in;
        } else {
            float* wf32 = static_cast<float*>(up(wh.data(), (size_t)nw * 4));
            f16* wf = static_cast<f16*>(dev((size_t)nw * 2));
            f32_to_f16(wf32, wf, nw, st);
            g.B1 = wf; g.ldb1 = in;
        }
        if (gemm_tc_supported(g)) {
            int sms = 0;
            LCK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
            g.sk_part = static_cast<float*>(dev(sizeof(float) * gemm_sk_part_floats(sms)));
            g.sk_flag = static_cast<int*>(dev(sizeof(int) * gemm_sk_flag_count(sms)));
            LCK(cudaMemsetAsync(g.sk_flag, 0, sizeof(int) * gemm_sk_flag_count(sms), st));
            gemm_tc_auto(g, derr, st);
        } else {
            gemm(g, st);
        }
        // the adapter (lora.h:56-79): reference order of operations, fp32
        const float s = adapted ? (dora ? alpha / rank : strength * alpha / rank) : 0.0f;
        const bool skip = !adapted || (dora ? strength == 0.0f : s == 0.0f);
        if (!skip) {
            const float* Ad = static_cast<const float*>(up(A, (size_t)rank * in * 4));
            const float* Bd = static_cast<const float*>(up(B, (size_t)out * rank * 4));
            float* U = static_cast<float*>(dev((size_t)rows * rank * 4));
            float* Yd = static_cast<float*>(dev((size_t)rows * out * 4));
            linear_f32(xd, Ad, U, (int)rows, rank, in, 0, st);   // U = x A^T
            linear_f32(U, Bd, Yd, (int)rows, out, rank, 0, st);  // B (A x)
            float* gd = nullptr;
            if (dora) {
                // ||W_o||^2 + in * 1e-12 in double from the bound values (lora_row_norm_sq)
                std::vector<float> nsq((size_t)out);
                for (int o = 0; o < out; ++o) {
                    double sum = in * 1e-12;
                    for (int i = 0; i < in; ++i) {
                        const float v = wh[(size_t)o * in + i];
                        if (!std::isfinite(v)) throw std::invalid_argument("nonfinite DoRA base weight");
                        sum += (double)v * v;
                    }
                    nsq[(size_t)o] = (float)sum;
                }
                const float* base = static_cast<const float*>(up(nsq.data(), (size_t)out * 4));
                const float* md = static_cast<const float*>(up(magnitude, (size_t)out * 4));
                const float* wd32 = static_cast<const float*>(up(wh.data(), (size_t)nw * 4));
                float* P = static_cast<float*>(dev((size_t)out * rank * 4));
                float* G = static_cast<float*>(dev((size_t)rank * rank * 4));
                linear_f32(wd32, Ad, P, out, rank, in, 0, st);  // W A^T
                linear_f32(Ad, Ad, G, rank, rank, in, 0, st);   // A A^T
                gd = static_cast<float*>(dev((size_t)out * 4));
                lora_dora_factor_kernel<<<(out + 127) / 128, 128, 0, st>>>(Bd, P, G, base, md, out, rank, s, gd);
            }
            const long n = rows * out;
            lora_combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(yd, Yd, n, out, s, gd, strength);
        }
        LCK(cudaGetLastError());
        LCK(cudaMemcpyAsync(y, yd, (size_t)rows * out * 4, cudaMemcpyDeviceToHost, st));
        int e = 0;
        LCK(cudaMemcpyAsync(&e, derr, sizeof(int), cudaMemcpyDeviceToHost, st));
        LCK(cudaStreamSynchronize(st));
        if (e) throw std::runtime_error("GEMM kernel reported a timed-out wait (code " + std::to_string(e) + ")");
    } catch (...) {
        cleanup();
        throw;
    }
    cleanup();
}

}  // namespace act

int act_lora_linear(int device, const float* x, int64_t rows, int in, int out, int w_type, const void* w,
                    size_t w_bytes, const float* A, const float* B, int rank, float alpha, const float* magnitude,
                    float strength, float* y) {
    try {
        act::lora_linear(device, x, rows, in, out, w_type, w, w_bytes, A, B, rank, alpha, magnitude, strength, y);
        return ACT_OK;
    } catch (const std::invalid_argument& e) {
        act::set_last_error(e.what());
        return ACT_ERR_INVALID;
    } catch (const std::exception& e) {
        act::set_last_error(e.what());
        return ACT_ERR_CUDA;
    }
}
