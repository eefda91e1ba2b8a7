// common.cuh -- shared device helpers for the adapter-training kernels (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

typedef __half f16;

namespace act {

// Kernel attributes set with cudaFuncSetAttribute belong to the device that is current at the
// call, so a one-time set-up has to run once on every device that launches the kernel.
// DeviceOnce runs its function at most once per device ordinal, from any number of host
// threads; ordinals beyond 63 run it on every call.
class DeviceOnce {
  public:
    template <class Fn>
    void operator()(Fn&& fn) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return;
        if (dev < 0 || dev >= 64) {
            fn();
            return;
        }
        const uint64_t bit = 1ull << dev;
        if (done_.load(std::memory_order_acquire) & bit) return;
        std::lock_guard<std::mutex> g(mu_);
        if (done_.load(std::memory_order_relaxed) & bit) return;
        fn();
        done_.fetch_or(bit, std::memory_order_release);
    }

  private:
    std::atomic<uint64_t> done_{0};
    std::mutex mu_;
};

// Multiprocessor count of the current device (cached per ordinal).
inline int current_sm_count() {
    static std::atomic<int> cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 1;
    int n = (dev >= 0 && dev < 64) ? cache[dev].load(std::memory_order_relaxed) : 0;
    if (n > 0) return n;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 1;
    if (dev >= 0 && dev < 64) cache[dev].store(n, std::memory_order_relaxed);
    return n;
}

// A&S 7.1.26 GELU and the derivative of that approximation (the reference trains through
// the approximation, src/ac/lora.h:97-110, so its gradient is the one autodiff yields).
// The reciprocal and exponential use the fast hardware approximations (relative error ~1e-6):
// every caller rounds the result to f16 (relative step 2^-8), and these run once per element
// of the widest GEMM epilogues.
__device__ __forceinline__ float gelu_as(float x) {
    const float z = x * 0.7071067811865475f, a = fabsf(z);
    const float t = __fdividef(1.0f, 0.3275911f * a + 1.0f);
    const float poly =
        ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
    const float e = __expf(-(z * z));
    const float sg = z > 0.f ? 1.f : (z < 0.f ? -1.f : 0.f);
    return x * (0.5f * (sg * (1.0f - poly * e)) + 0.5f);
}

__device__ __forceinline__ float gelu_as_grad(float x) {
    const float z = x * 0.7071067811865475f, a = fabsf(z);
    const float sg = z > 0.f ? 1.f : (z < 0.f ? -1.f : 0.f);
    const float t = __fdividef(1.0f, 0.3275911f * a + 1.0f);
    const float poly =
        ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
    const float dpoly =
        (((5.0f * 1.061405429f * t - 4.0f * 1.453152027f) * t + 3.0f * 1.421413741f) * t - 2.0f * 0.284496736f) * t +
        0.254829592f;
    const float e = __expf(-(z * z));
    const float erf_ = sg * (1.0f - poly * e);
    const float derf = sg * sg * dpoly * 0.3275911f * t * t * e + 2.0f * z * sg * poly * e;
    return (0.5f * erf_ + 0.5f) + x * 0.5f * derf * 0.7071067811865475f;
}

// gelu_as(x) and gelu_as_grad(x) from one evaluation of the shared terms.  sg(z)^2 = 1 is used
// in the derivative: it differs only at z = 0, where that term is multiplied by x = 0.
__device__ __forceinline__ void gelu_as_pair(float x, float& g, float& dg) {
    const float z = x * 0.7071067811865475f, a = fabsf(z);
    const float t = __fdividef(1.0f, 0.3275911f * a + 1.0f);
    const float poly =
        ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
    const float dpoly =
        (((5.0f * 1.061405429f * t - 4.0f * 1.453152027f) * t + 3.0f * 1.421413741f) * t - 2.0f * 0.284496736f) * t +
        0.254829592f;
    const float e = __expf(-(z * z));
    const float pe = poly * e;
    const float half_cdf = 0.5f * copysignf(1.0f - pe, z) + 0.5f;
    g = x * half_cdf;
    const float derf = dpoly * 0.3275911f * t * t * e + 2.0f * a * pe;
    dg = half_cdf + x * 0.5f * derf * 0.7071067811865475f;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
    const int bytes = pred ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem),
                 "r"(bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                        const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                          const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}

// D += A(16x16, row) * B(16x8, col), f16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_sync_f16(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// two floats rounded to nearest-even f16, lo in the low half-word
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// the two f16 halves of a word as floats
__device__ __forceinline__ float2 unpack_f16(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}


// ---------------------------------------------------------------------------------------
// Programmatic dependent launch: a kernel launched with the programmatic-serialization attribute
// may start while its predecessor drains; it runs its prologue (barriers, TMEM, descriptors),
// then waits here before touching memory the predecessor writes.  Every kernel lets its
// successor start early (the successor still waits for this grid's completion).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline void pdl_attr(cudaLaunchAttribute& at) {
    at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at.val.programmaticStreamSerializationAllowed = 1;
}

// Launch a kernel that starts with pdl_wait() with the programmatic-serialization attribute.
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    pdl_attr(attr[0]);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace act
