// attention_noalloc.cu -- attention backward for callers that cannot allocate device memory.
//
// Some callers of this library must not call cudaMalloc or cudaFree:
//   * a real-time host such as an audio plug-in's processing thread, where an allocation can
//     block for milliseconds and implicitly synchronise the device, breaking its deadline;
//   * code that records work into a CUDA graph under global stream capture, where cudaMalloc
//     is not permitted at all;
//   * an embedder that owns every device byte through its own memory pool and does not let
//     libraries allocate behind its back.
// act_attention_bwd_noalloc gives them the attention backward with no allocation: they pass
// their own inputs and outputs, and the scratch the backward needs (the fp32 dQ accumulator
// and the per-row rowsum(dO * O) vector) lives in a fixed array compiled into this library.
#include <mutex>
#include <string>

#include "actrain.h"
#include "kernels.h"

namespace {

// Fixed scratch: ACT_NOALLOC_ATTN_SCRATCH_FLOATS floats (32 MiB).  Every GPU that loads this
// library holds it until the process exits.  All calls share it.
static __device__ __align__(256) float g_attn_scratch[ACT_NOALLOC_ATTN_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
float* g_scratch_ptr[kMaxDevices] = {};

int fail(int code, const std::string& msg) {
    act::set_last_error(msg);
    return code;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int attention_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const float* lse,
                          const void* dout, void* dq, void* dk, void* dv, int clips, int T, int Tk, int H,
                          const int32_t* nvalid, int causal, int zero_key, const float* rope, void* stream) {
    if (!q || !k || !v || !o || !lse || !dout || !dq || !dk || !dv)
        return fail(ACT_ERR_INVALID, "act_attention_bwd_noalloc: null pointer");
    if (clips <= 0 || T <= 0 || Tk <= 0 || H <= 0)
        return fail(ACT_ERR_INVALID, "act_attention_bwd_noalloc: sizes must be positive");
    if (causal && Tk != T) return fail(ACT_ERR_INVALID, "act_attention_bwd_noalloc: causal attention needs Tk == T");
    if (rope && Tk > T) return fail(ACT_ERR_INVALID, "act_attention_bwd_noalloc: RoPE needs Tk <= T");
    // The kernels move the f16 tensors in 16-byte vectors, the RoPE table in (cos, sin) float
    // pairs and lse / nvalid as 4-byte words: a misaligned pointer would fault on the device, so
    // it is rejected here, before anything is queued.
    for (const void* p : {q, k, v, o, dout, static_cast<const void*>(dq), static_cast<const void*>(dk),
                          static_cast<const void*>(dv)})
        if (!aligned(p, 16))
            return fail(ACT_ERR_INVALID, "act_attention_bwd_noalloc: q, k, v, o, dout, dq, dk and dv must be "
                                         "16-byte aligned");
    if (!aligned(lse, 4) || (nvalid && !aligned(nvalid, 4)) || (rope && !aligned(rope, 8)))
        return fail(ACT_ERR_INVALID, "act_attention_bwd_noalloc: lse and nvalid must be 4-byte aligned, rope "
                                     "8-byte aligned");
    const long D = (long)H * 64;
    const long acc_floats = (long)clips * T * D;          // dQ accumulator
    const long dvec_floats = (long)clips * H * T;         // rowsum(dO * O)
    const long need = acc_floats + dvec_floats;
    if (need > (long)ACT_NOALLOC_ATTN_SCRATCH_FLOATS)
        return fail(ACT_ERR_INVALID, "act_attention_bwd_noalloc: this problem needs " + std::to_string(need) +
                                         " floats of scratch; the fixed maximum is " +
                                         std::to_string((long)ACT_NOALLOC_ATTN_SCRATCH_FLOATS) +
                                         " (clips * T * H * 64 + clips * H * T)");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(ACT_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(ACT_ERR_INVALID, "act_attention_bwd_noalloc: device ordinal out of range");
    float* scratch = nullptr;
    {
        // One-time set-up per device, with that device current: the address of this device's copy
        // of the array.  The host-side symbol is only a stand-in and must never reach a kernel.
        // The address is kept for the life of the process, so the device must not be reset
        // (cudaDeviceReset, or a reset of its primary context) after the first call.
        std::lock_guard<std::mutex> lock(g_scratch_mu);
        if (!g_scratch_ptr[dev]) {
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, g_attn_scratch);
            if (e != cudaSuccess || !p)
                return fail(ACT_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
            g_scratch_ptr[dev] = static_cast<float*>(p);
        }
        scratch = g_scratch_ptr[dev];
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    act::AttnArgs a;
    a.q = static_cast<const f16*>(q);
    a.k = static_cast<const f16*>(k);
    a.v = static_cast<const f16*>(v);
    a.ldq = a.ldk = a.ldv = D;
    a.T = T; a.Tk = Tk; a.H = H; a.clips = clips;
    a.nvalid = nvalid;
    a.causal = causal;
    a.zero_key = zero_key;
    a.rope = rope;
    a.rope_load = 1;
    a.scale = 0.125f;
    a.o = const_cast<f16*>(static_cast<const f16*>(o));
    a.ldo = D;
    a.lse = const_cast<float*>(lse);
    a.dout = static_cast<const f16*>(dout);
    a.lddo = D;
    a.dq_acc = scratch;                 // accumulated with atomics: must start at zero every call
    a.ldq_acc = D;
    a.dvec = scratch + acc_floats;      // fully overwritten every call
    a.dk = static_cast<f16*>(dk);
    a.dv = static_cast<f16*>(dv);
    a.lddk = a.lddv = D;
    e = cudaMemsetAsync(a.dq_acc, 0, sizeof(float) * acc_floats, st);
    if (e != cudaSuccess) return fail(ACT_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
    act::attn_bwd(a, st);
    act::attn_dq_finish(a, static_cast<f16*>(dq), D, nullptr, st);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail(ACT_ERR_CUDA, std::string("attention backward launch: ") + cudaGetErrorString(e));
    return ACT_OK;
}

}  // namespace

extern "C" int act_attention_bwd_noalloc(const void* q, const void* k, const void* v, const void* o,
                                         const float* lse, const void* dout, void* dq, void* dk, void* dv,
                                         int clips, int T, int Tk, int H, const int32_t* nvalid, int causal,
                                         int zero_key, const float* rope, void* stream) {
    // no C++ exception may cross the C ABI: an embedding host would terminate
    try {
        return attention_bwd_noalloc(q, k, v, o, lse, dout, dq, dk, dv, clips, T, Tk, H, nvalid, causal, zero_key,
                                     rope, stream);
    } catch (const std::exception& ex) {
        try {
            return fail(ACT_ERR_INVALID, std::string("act_attention_bwd_noalloc: ") + ex.what());
        } catch (...) {
            return ACT_ERR_INVALID;
        }
    } catch (...) {
        return ACT_ERR_INVALID;
    }
}
