// Device helpers shared by the attention kernels (sm_100a): shared-memory barriers with bounded
// waits, CTA-local TMA tile loads, ldmatrix / mma.sync fragments, and the
// 128-byte swizzle that TMA applies to [rows][64 x fp16] boxes.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace brk {

// Every spin on a barrier gives up after kWaitNs of wall time (read from %globaltimer) or
// kWaitPolls polls, whichever comes first, records a timeout in the context's error word and
// lets the kernel finish without the data.  Legitimate waits last microseconds.
constexpr unsigned long long kWaitNs = 2000000000ull;
constexpr uint32_t kWaitPolls = 1u << 28;

enum DeviceError : int {
    kErrNone = 0,
    kErrTmaTimeout = 1,   // a consumer waited too long for a TMA tile
    kErrSlotTimeout = 2,  // the producer waited too long for a free ring slot
    kErrMmaTimeout = 3,   // a tcgen05 commit never arrived
    kErrPeerTimeout = 4,  // a rank's partials never arrived (sequence-sharded combine)
};

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes barrier initialisation visible to the async (TMA / tensor core) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Orders this thread's generic-proxy global stores before later async-proxy (TMA) accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for phase `parity` of `bar`.  On timeout writes `code` into *err (first error
// wins) and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_timer_ns();
    for (uint32_t i = 1; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0 && global_timer_ns() - t0 > kWaitNs) break;
    }
    if (err) atomicCAS(err, 0, code);
    return false;
}

// 2-D tiled TMA load (into this CTA only) of the box at (x = column, y = row) into shared memory,
// completing `bar`'s transaction count.  x * sizeof(element) must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a [rows][128 B] box written by
// TMA with CU_TENSOR_MAP_SWIZZLE_128B into a 1024-byte aligned buffer: chunk index XOR row%8.
__device__ __forceinline__ uint32_t sw128(uint32_t row, uint32_t chunk) {
    return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// Same for a [rows][64 B] box written with CU_TENSOR_MAP_SWIZZLE_64B into a 512-byte aligned
// buffer: chunk (0..3) XOR address bits 7-8, i.e. (row / 2) % 4.
__device__ __forceinline__ uint32_t sw64(uint32_t row, uint32_t chunk) {
    return row * 64u + ((chunk ^ ((row >> 1) & 3u)) << 4);
}

// Byte permute: byte i of the result is byte sel[4i+3:4i] of the 8-byte value {b, a}.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// Two int8 KV codes stored biased (u = code + 128, one byte each) -> fp16x2 of code + 1152,
// exactly.  `sel` picks the two bytes of w into bytes 0 and 2 of the fp16 pair (0x4140: bytes
// 0, 1; 0x4342: bytes 2, 3); bytes 1 and 3 become 0x64, so each half reads 1024 + u = 1152 + code
// (0x64uu is exponent 10 with u in the low mantissa bits).  Users subtract kCodeBias * (sum of
// the other operand) from their dot products instead of 1152 from every code.
constexpr float kCodeBias = 1152.f;
__device__ __forceinline__ uint32_t codes_biased_half2(uint32_t w, uint32_t sel) { return prmt(w, 0x64646464u, sel); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D = A(16x16, row) * B(16x8, col) + D, fp16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Transpose of an 8x8 fp16 matrix held as an mma fragment (lane l: row l/4, columns 2(l%4) and
// 2(l%4)+1): returns the same fragment of the transposed matrix.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

// Hardware 2^x (MUFU; ~2 ulp, flushes subnormals; 2^-inf = 0), for softmax probabilities.
__device__ __forceinline__ float ex2_fast(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Hardware reciprocal (MUFU; ~1 ulp, flushes subnormals; 1/inf = 0).
__device__ __forceinline__ float rcp_fast(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Logit softcap c * tanh(s / c) (shaders.ts:1490) in log2 units, from tanh(z) = 1 - 2 / (1 + e^{2z})
// with k1 = 2 * scale * log2(e) / c and k2 = c * log2(e): one MUFU exponential and one MUFU
// reciprocal, saturating to +-k2 for large |z|.  The tanh comes out within a few 1e-7 absolute
// (near z = 0 the subtraction cancels, which costs relative but not absolute precision).
__device__ __forceinline__ float softcap_log2(float s, float k1, float k2) {
    return k2 * (1.f - 2.f * rcp_fast(1.f + ex2_fast(s * k1)));
}

// Three-input maximum (one instruction on sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Maximum of N registers as a tree of three-input maxima (depth log3 N instead of a chain of N).
template <int N>
__device__ __forceinline__ float max_tree(const float (&v)[N]) {
    constexpr int M = (N + 2) / 3;
    float w[M];
#pragma unroll
    for (int i = 0; i < M; ++i) {
        if (3 * i + 2 < N)
            w[i] = fmax3(v[3 * i], v[3 * i + 1], v[3 * i + 2]);
        else if (3 * i + 1 < N)
            w[i] = fmaxf(v[3 * i], v[3 * i + 1]);
        else
            w[i] = v[3 * i];
    }
    if constexpr (M == 1)
        return w[0];
    else
        return max_tree<M>(w);
}

// Two lanes of f32 arithmetic in one instruction (sm_100 packed f32x2); each lane rounds like
// the scalar fmaf / add.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 pa, pb, pc, pd;\n\t"
        "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\tmov.b64 pc, {%6, %7};\n\t"
        "fma.rn.f32x2 pd, pa, pb, pc;\n\tmov.b64 {%0, %1}, pd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 pa, pb, pd;\n\t"
        "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
        "add.rn.f32x2 pd, pa, pb;\n\tmov.b64 {%0, %1}, pd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// 2^x for two lanes on the FMA pipe, for softmax probabilities that end up as fp16.  The method
// is the textbook range reduction of exp2 (as in Cody and Waite's elementary-function
// algorithms) followed by a minimax-style polynomial: x = n + f with n = round(x) (adding and
// subtracting 1.5 * 2^23), f in [-0.5, 0.5]; 2^f from a cubic fitted here to 2^f on
// [-0.5, 0.5] by relative-error least squares (max relative error 1.0e-4, below half an fp16
// ulp); n added to the exponent field.  x is clamped at -127 (result 0).
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
    constexpr float kShift = 12582912.f;  // 1.5 * 2^23
    x.x = fmaxf(x.x, -127.f);
    x.y = fmaxf(x.y, -127.f);
    const float2 j = fadd2(x, make_float2(kShift, kShift));
    const float2 n = fadd2(j, make_float2(-kShift, -kShift));
    const float2 f = fadd2(x, make_float2(-n.x, -n.y));
    float2 p = ffma2(make_float2(0.05500883609056473f, 0.05500883609056473f), f,
                     make_float2(0.24221085011959076f, 0.24221085011959076f));
    p = ffma2(p, f, make_float2(0.6932829022407532f, 0.6932829022407532f));
    p = ffma2(p, f, make_float2(1.f, 1.f));
    // The low bits of j hold n (two's complement); shifted into the exponent field.
    return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(j.x) << 23)),
                       __int_as_float(__float_as_int(p.y) + (__float_as_int(j.y) << 23)));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

// Programmatic dependent launch: wait for the grids this one depends on (completion and memory
// visibility); a no-op when the launch has no programmatic dependency.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Lets the next programmatic-dependent grid in the stream be scheduled.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// System-scope release store / acquire load of a 32-bit flag (the flag may live in another GPU's
// memory mapped into this process).
__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Thread-block cluster barrier (every thread of every CTA of the cluster arrives, release /
// acquire at cluster scope), in the non-aligned form so that diverged warps may take it.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// f32 at the same shared-memory offset as `p` in CTA `rank` of this cluster (distributed shared
// memory).
__device__ __forceinline__ float ld_cluster_f32(const float *p, unsigned rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(p)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace brk
