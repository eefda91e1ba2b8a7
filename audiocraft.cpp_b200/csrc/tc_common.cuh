// tc_common.cuh -- PTX helpers shared by the tcgen05 kernels (sm_100a): bounded mbarrier waits,
// TMA tile loads, UMMA shared-memory descriptors, tcgen05.mma / commit / ld, and the host-side
// tensor-map encoder.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace act {
namespace tc {

constexpr unsigned long long WAIT_NS = 2000000000ull;  // 2 s per wait

// Instruction-descriptor bits shared by every tcgen05.mma.kind::f16 here: fp32 accumulator
// (bits 4-5 = 1) with f16 A and B operands (bits 7-9 and 10-12 = 0).  Majors, N >> 3 and
// M >> 4 are or-ed in per call site.
constexpr uint32_t IDESC_F16_F32ACC = 1u << 4;

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase completes or the hint
// (nanoseconds) expires, instead of polling and taking issue slots from the warps that work
__device__ __forceinline__ bool mbar_try_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait: returns false (and records `code`) if the phase does not complete in time.
// The first probe is inline (the common case on the issue paths); the sleeping loop is not.
static __device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, int* err, int code) {
    const unsigned long long t0 = globaltimer();
    while (true) {
        for (int i = 0; i < 16; ++i)
            if (mbar_try_sleep(bar, parity, 100000u)) return true;
        if (globaltimer() - t0 > WAIT_NS) {
            atomicCAS(err, 0, code);
            return false;
        }
        if (*(volatile int*)err) return false;  // another CTA already failed: stop waiting
    }
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
    return mbar_try(bar, parity) || mbar_wait_slow(bar, parity, err, code);
}

// Wait for copies this thread issued to land before its CTA exits, after another wait failed:
// bounded (limit_ns) but not cut short by the error word, which is already set by then.
static __device__ __noinline__ void mbar_wait_drain(uint32_t bar, uint32_t parity,
                                                    unsigned long long limit_ns = 100000000ull) {
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_sleep(bar, parity, 20000u))
        if (globaltimer() - t0 > limit_ns) return;
}

// Global flags between CTAs of one grid (all co-resident): release add by the producer side,
// bounded acquire poll by the consumer side.
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add(int* p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until *flag >= target; false (and `code` recorded) if that does not happen within
// limit_ns nanoseconds.
static __device__ __noinline__ bool flag_wait(const int* flag, int target, int* err, int code,
                                              unsigned long long limit_ns = WAIT_NS) {
    const unsigned long long t0 = globaltimer();
    while (ld_acquire_gpu(flag) < target) {
        __nanosleep(256);
        if (globaltimer() - t0 > limit_ns) {
            atomicCAS(err, 0, code);
            return false;
        }
        if (*(volatile int*)err) return false;
    }
    return true;
}

// Contiguous global -> shared copy by the bulk-copy engine (16-byte aligned, size % 16 == 0),
// completing on an mbarrier of this CTA.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Fetch a tensor map (kernel parameter) into the descriptor cache ahead of its first use; issued
// before the programmatic-dependent-launch wait, it overlaps the previous kernel's tail.
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
    d |= 1ull << 46;  // descriptor version (sm100)
    d |= 2ull << 61;  // SWIZZLE_128B
    return d;
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------------------
// Q8_0 weights dequantised in shared memory on their way into an MMA operand (the 2-CTA GEMM's
// B and the rank-block kernel's A): a raw slot holds one k-block of biased quants (q + 128) and
// their f16 block scales as TMA brought them; converter threads write the f16 operand tile in
// the 128-byte-swizzled layout a TMA load of the f16 values would have produced.
constexpr int Q8_BK = 64;  // k per block of the operand ring

// byte offset of 16-byte unit u of row r in a 128-byte-swizzled tile (1024-byte aligned)
__device__ __forceinline__ uint32_t q8_sw128(int r, int u) { return r * 128 + ((u ^ (r & 7)) << 4); }

// Eight Q8_0 quants (biased: q + 128, one byte each) times their block scale -> eight f16.  The
// biased quant goes into the mantissa of the f16 1024 + (q + 128) (byte permute), 1152 is
// subtracted (exact), and one f16 multiply rounds q * d to nearest-even: the same single rounding
// of the exact product that the bind-time dequantisation applies (fp32 d * q, exact, to f16).
__device__ __forceinline__ uint4 q8x8_to_f16(uint2 u, uint32_t dd) {
    const uint32_t w[4] = {__byte_perm(u.x, 0x64646464u, 0x5140), __byte_perm(u.x, 0x64646464u, 0x5342),
                           __byte_perm(u.y, 0x64646464u, 0x5140), __byte_perm(u.y, 0x64646464u, 0x5342)};
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    const __half2 d2 = *reinterpret_cast<const __half2*>(&dd);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 v = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&w[i]), bias), d2);
        o[i] = *reinterpret_cast<const uint32_t*>(&v);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// One k-block of Q8_0 B for this CTA into its f16 operand slot, by NT converter threads (ct).
// K-major (forward, B(n, k) = W[n][k]): raw quants [BH][64] bytes, scales [2][BH] (k / 32, n);
// the operand is rows of 128 bytes with the 128-byte swizzle TMA would have applied.
// MN-major (input gradient, B(n, k) = W[k][n]): raw quants [64][BH] bytes, scales [BH / 32][64]
// (n / 32, k); the operand is BH / 64 boxes of [64 k][64 n] with the same swizzle.  Lanes read
// consecutive 8-byte pieces of a row (conflict-free) and write whole swizzled 128-byte rows.
template <int BH, bool B_MN, int NT>
__device__ __forceinline__ void convert_q8_stage(const unsigned char* smem, uint32_t rq_off, uint32_t sb_off, int ct) {
    const unsigned char* rq = smem + rq_off;
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(rq + BH * Q8_BK);
    unsigned char* sb = const_cast<unsigned char*>(smem) + sb_off;
    // Every load of the k-block is issued before the first store: the compiler cannot tell the
    // raw slot from the operand tile, so interleaved loads and stores would each wait for the
    // shared-memory latency (long while the tensor core streams its operands).
    if (!B_MN) {
        constexpr int RPP = NT / 8;  // rows per pass: 8 chunks of 8 k per row
        constexpr int IT = BH / RPP;
        uint2 q[IT];
        uint32_t d[IT];
        const int c = ct & 7;
#pragma unroll
        for (int it = 0; it < IT; ++it) {
            const int row = it * RPP + (ct >> 3);
            q[it] = *reinterpret_cast<const uint2*>(rq + row * Q8_BK + c * 8);
            d[it] = sc[(c >> 2) * BH + row];
        }
#pragma unroll
        for (int it = 0; it < IT; ++it) {
            const int row = it * RPP + (ct >> 3);
            *reinterpret_cast<uint4*>(sb + q8_sw128(row, c)) = q8x8_to_f16(q[it], d[it] | (d[it] << 16));
        }
    } else {
        constexpr int CPR = BH / 8;    // 8-wide chunks of n per k-row
        constexpr int RPP = NT / CPR;  // k-rows per pass
        constexpr int IT = Q8_BK / RPP;
        uint2 q[IT];
        uint32_t d[IT];
        const int c = ct % CPR;
#pragma unroll
        for (int it = 0; it < IT; ++it) {
            const int k = it * RPP + ct / CPR;
            q[it] = *reinterpret_cast<const uint2*>(rq + k * BH + c * 8);
            d[it] = sc[(c >> 2) * Q8_BK + k];
        }
#pragma unroll
        for (int it = 0; it < IT; ++it) {
            const int k = it * RPP + ct / CPR;
            *reinterpret_cast<uint4*>(sb + (c >> 3) * 8192 + q8_sw128(k, c & 7)) =
                q8x8_to_f16(q[it], d[it] | (d[it] << 16));
        }
    }
}

}  // namespace tc


// Host: cuTensorMapEncodeTiled through the driver entry point (no libcuda link dependency).
// 2D f16 row-major tensor [rows][cols] with row stride ld (elements); box {box_cols, box_rows},
// 128-byte swizzle.
void tc_make_map(CUtensorMap* map, const f16* ptr, long rows, long cols, long ld, int box_cols, int box_rows);
// Unswizzled map of raw bytes (f16v = 0: uint8 Q8_0 quants) or f16 values (f16v = 1: their block
// scales), [rows][cols] with row stride ld elements, box {box_cols, box_rows}.
void tc_make_map_raw(CUtensorMap* map, const void* ptr, bool f16v, long rows, long cols, long ld, int box_cols,
                     int box_rows);
// 3-D f16 tensor [clips][rows][cols] (row stride ld elements, clip stride rows * ld): a box
// {box_cols, box_rows, 1} never crosses into the next clip (rows past `rows` read as zero).
void tc_make_map3(CUtensorMap* map, const f16* ptr, long clips, long rows, long cols, long ld, int box_cols,
                  int box_rows);

}  // namespace act
