// Shared device helpers for the AudioVAE decoder kernels (sm_100a only).
//
// PTX wrappers for mbarriers, TMA tile loads, TMEM allocation, tcgen05.mma and
// tcgen05.ld, plus the bounded waits every kernel uses: a wait that does not
// complete within kWaitNs nanoseconds records an error code in the plan's
// device status word and makes the kernel bail out instead of spinning
// forever.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "these kernels target sm_100a only"
#endif

namespace vxb {

// Error codes written to the device status word (first writer wins).
enum DevStatus : int {
    kOk = 0,
    kErrWaitFull = 1,      // MMA issuer gave up waiting for a loaded stage
    kErrWaitEmpty = 2,     // producer gave up waiting for a free stage
    kErrWaitAccum = 3,     // epilogue gave up waiting for the accumulator
    kErrBadLaunch = 4,     // launch geometry did not match the kernel's contract
};

constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s per wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void set_status(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

// ------------------------------------------------------------- mbarrier --

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One try with a suspend-time hint: the thread sleeps (without issuing) until
// the phase completes or about 20 us pass, so waiting warps do not take
// issue slots from the working ones.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "n"(20000)
        : "memory");
    return ok != 0;
}

// Bounded wait on a phase of an mbarrier.  Returns false (and records `code`)
// when the phase has not completed within kWaitNs, or when another role of
// the CTA has already aborted (*abort != 0).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* status,
                                          int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (globaltimer_ns() - t0 > kWaitNs) {
            *abort = 1;
            set_status(status, code);
            return false;
        }
    }
}

// The same bounded wait with the limit given in nanoseconds (the failure
// probe waits on a barrier nothing arrives on, with a short limit).
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, volatile int* abort, int* status,
                                              int code, unsigned long long limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (globaltimer_ns() - t0 > limit_ns) {
            *abort = 1;
            set_status(status, code);
            return false;
        }
    }
}

// ------------------------------------------------ programmatic launches --
// Every decode kernel is launched with programmatic stream serialisation:
// it may start (and run its setup) while the previous kernel finishes, and
// waits here before touching memory the previous kernels wrote or read.
// griddepcontrol.wait returns once every prerequisite grid has completed and
// its memory operations are visible; launch_dependents then lets the next
// kernel be scheduled (issued only after the wait, so at most two grids are
// in flight).  Without a programmatic prerequisite both are no-ops.
__device__ __forceinline__ void grid_dep_sync() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// -------------------------------------------------------------------- TMA --

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(smem_dst)), "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// L2 prefetch of a 2-D tensor-map box: no shared memory, no completion.
__device__ __forceinline__ void tma_prefetch_2d(const void* tmap, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(tmap), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(smem_u32(smem_dst)), "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// Shared -> global tile store (bulk-group completion), and its waits.
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* smem_src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(tmap), "r"(smem_u32(smem_src)), "r"(x), "r"(y)
                 : "memory");
}

// One 32-byte global store (sm_100: st.global.v8; p 32-byte aligned).
__device__ __forceinline__ void st_global_v8(float* p, const float4& a, const float4& b) {
    asm volatile("st.global.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "f"(a.x), "f"(a.y), "f"(a.z),
                 "f"(a.w), "f"(b.x), "f"(b.y), "f"(b.z), "f"(b.w)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* smem_src, int x, int y, int z) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
                 ::"l"(tmap), "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z)
                 : "memory");
}

// Waits until at most N committed bulk groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Waits until every committed bulk group has completed (writes visible).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 16-byte global -> shared copy (cp.async, cached at L2 only); src_bytes = 0
// writes zeros without reading src.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// Pulls the 128-byte line holding p into L2 (no register result).
__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p) : "memory");
}

// Makes generic-proxy shared-memory writes visible to the async proxy
// (tcgen05.mma reads operands through it).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Named barrier `id` over one 128-thread epilogue warpgroup.
__device__ __forceinline__ void epi_bar(int id) { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }

// The same barrier, also OR-ing a predicate: true on every thread if any
// thread passed true (a uniform bail-out).
__device__ __forceinline__ bool epi_bar_any(int id, bool p) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %2, 0;\n barrier.red.or.pred q, %1, 128, p;\n"
        " selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"(id), "r"(static_cast<uint32_t>(p))
        : "memory");
    return r != 0;
}

// ------------------------------------------------------------------- TMEM --

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (fp16 inputs, fp32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on `bar` when all previously issued tcgen05.mma of this thread
// have completed (frees a smem stage / publishes the accumulator).
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 32 lanes x 16 consecutive fp32 columns; thread i of the warp gets lane
// (warp's quadrant base + i), columns col..col+15.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ------------------------------------------------------- UMMA descriptors --
// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"):
//   [0,14) start address >> 4, [16,30) leading byte offset >> 4,
//   [32,46) stride byte offset >> 4, [46,48) version = 1,
//   [49,52) base offset = 0, [52] LBO mode = 0, [61,64) swizzle (2 = 128 B).
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;
    d |= 2ull << 61;
    return d;
}

// Instruction descriptor, kind::f16: D fp32, A and B fp16, dense.
//   [4,6) D format (1 = f32), [7,10) A format (0 = f16), [10,13) B format,
//   [15] A major (0 = K, 1 = MN), [16] B major, [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N, int a_mn_major) {
    return (1u << 4) | (static_cast<uint32_t>(a_mn_major) << 15) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// Byte offset of element (row, k) in a K-major tile of 128-byte rows with the
// 128-byte swizzle (8-row atoms of 1024 B, 16-byte chunk index XOR row%8):
// the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B and the one the
// K-major SW128 descriptor reads.
__device__ __forceinline__ uint32_t sw128_kmajor_off(uint32_t row, uint32_t k) {
    return (row >> 3) * 1024u + (row & 7u) * 128u + ((((k >> 3) ^ row) & 7u) << 4) + (k & 7u) * 2u;
}

// ------------------------------------------------------------------ math --

// sin(a)^2.  sin^2 has period pi, so a is reduced to r = a - k*pi with k the
// integer nearest a/pi, |r| <= pi/2 (Cody-Waite: pi = hi + lo, hi = 201/64;
// fmaf keeps k*hi exact), and the hardware sine (__sinf, absolute error
// below 2^-21.41 on [-pi, pi]) is squared.  k is rounded on the FMA pipe:
// adding 1.5 * 2^23 leaves the nearest integer in the significand (exact for
// |a/pi| < 2^22).  The reduction adds less than 2e-7 + 2e-11*|a| of phase
// error, so sin^2 is off by less than 1.2e-6 + 4e-11*|a|, and Snake's
// y = x + inv * sin^2(alpha * x) by less than inv * 1.2e-6 + |x| * 2^-23
// (the last term includes rounding alpha * x).  For |a| >= 2^22 * pi any
// value of sin^2 in [0, 1] is within inv <= |x| * 2^-22 of the true one, so
// the bound inv * 1.2e-6 + |x| * 2^-22 holds for every x.  No branch.
constexpr double kPi = 3.14159265358979323846;
constexpr float kPiHi = 3.140625f;  // 201/64
constexpr float kPiLo = static_cast<float>(kPi - 3.140625);
constexpr float kInvPi = static_cast<float>(1.0 / kPi);
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23

__device__ __forceinline__ float sin_sq(float a) {
    const float k = fmaf(a, kInvPi, kRoundMagic) - kRoundMagic;
    float r = fmaf(-k, kPiHi, a);
    r = fmaf(-k, kPiLo, r);
    const float s = __sinf(r);
    return s * s;
}

// Eight Q4_0 values -> eight fp16 (one 16-byte smem chunk), (q - 8) * d.
// w0, w1 hold the 8 bytes whose low (hi = false) or high (hi = true)
// nibbles are the values, in order.  Each nibble q is OR-ed into the fp16
// pattern of 1024 (0x6400), giving 1024 + q exactly; subtracting 1032
// gives q - 8 exactly, and one fp16 multiply by d rounds the exact product
// (at most 15 significant bits) once -- the same result as rounding the
// fp32 product (q - 8) * d to fp16.
__device__ __forceinline__ uint4 q4_dequant8(uint32_t w0, uint32_t w1, bool hi, __half2 d2) {
    const uint32_t a0 = hi ? (w0 >> 4) : w0;
    const uint32_t a1 = hi ? (w1 >> 4) : w1;
    uint32_t p[4];
    p[0] = (a0 & 0x0000000Fu) | ((a0 << 8) & 0x000F0000u);
    p[1] = ((a0 >> 16) & 0x0000000Fu) | ((a0 >> 8) & 0x000F0000u);
    p[2] = (a1 & 0x0000000Fu) | ((a1 << 8) & 0x000F0000u);
    p[3] = ((a1 >> 16) & 0x0000000Fu) | ((a1 >> 8) & 0x000F0000u);
    const __half2 k1032 = __float2half2_rn(1032.0f);
    uint4 out;
    uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t bits = p[i] | 0x64006400u;
        __half2 h = *reinterpret_cast<const __half2*>(&bits);
        h = __hmul2(__hsub2(h, k1032), d2);
        o[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return out;
}

// The nibble order of the GEMMs' split Q4_0 weights: one 32-bit word holds
// the 8 values v0..v7 of a 16-byte smem chunk with v(i) in nibble slot
// kQ4Slot[i] (slot n = bits 4n..4n+3), so that masking the word shifted by
// 4j with 0x000F000F picks the pair (v2j, v2j+1) into the two halves.
__host__ __device__ constexpr int q4_slot(int i) { return (i & 1) * 4 + (i >> 1); }

// One word of the split layout -> eight fp16 (one 16-byte smem chunk),
// (q - 8) * d: each pair's nibbles are OR-ed into the fp16 pattern of 1024
// (0x6400) in one lop3, giving 1024 + q exactly; subtracting 1032 gives
// q - 8 exactly and one fp16 multiply by d rounds the exact product once --
// the same value as rounding the fp32 product (q - 8) * d to fp16.
__device__ __forceinline__ uint4 q4_dequant8_split(uint32_t w, __half2 d2) {
    const __half2 k1032 = __float2half2_rn(1032.0f);
    uint4 out;
    uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t bits;
        asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(bits) : "r"(w >> (4 * j)), "r"(0x000F000Fu), "r"(0x64006400u));
        __half2 h = *reinterpret_cast<const __half2*>(&bits);
        h = __hmul2(__hsub2(h, k1032), d2);
        o[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return out;
}

// Snake activation (reference audio-vae.cpp:278-289 / :1443-1479):
// x + sin(alpha*x)^2 * inv, inv = 1 / (alpha + 1e-9).
__device__ __forceinline__ float snake(float x, float alpha, float inv) {
    return fmaf(sin_sq(alpha * x), inv, x);
}

// ----------------------------------------------- paired fp32 arithmetic --
// sm_100 executes two fp32 FMAs / multiplies as one instruction
// (fma.rn.f32x2, mul.rn.f32x2; same IEEE rounding per lane as fmaf / fmul).
__device__ __forceinline__ uint64_t f2_bits(float2 a) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a.x), "f"(a.y));
    return r;
}
__device__ __forceinline__ float2 f2_val(uint64_t r) {
    float2 a;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a.x), "=f"(a.y) : "l"(r));
    return a;
}
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
    return f2_val(d);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_val(d);
}

// Snake on two lanes at once: the same operations and roundings as snake()
// per lane (alpha*x, the period-pi reduction, the hardware sine, the square
// and the final fma), paired where sm_100 has a two-lane instruction
// (-k = M - (a/pi + M) is exact, as is k = (a/pi + M) - M).
__device__ __forceinline__ float2 snake2(float2 x, float2 alpha, float2 inv) {
    const float2 a = fmul2(alpha, x);
    const float2 t = ffma2(a, make_float2(kInvPi, kInvPi), make_float2(kRoundMagic, kRoundMagic));
    const float2 k = ffma2(t, make_float2(-1.f, -1.f), make_float2(kRoundMagic, kRoundMagic));  // -nearest(a/pi)
    float2 r = ffma2(k, make_float2(kPiHi, kPiHi), a);
    r = ffma2(k, make_float2(kPiLo, kPiLo), r);
    const float2 sn = make_float2(__sinf(r.x), __sinf(r.y));
    return ffma2(fmul2(sn, sn), inv, x);
}

__device__ __forceinline__ float4 snake4(float4 x, float4 alpha, float4 inv) {
    const float2 lo = snake2(make_float2(x.x, x.y), make_float2(alpha.x, alpha.y), make_float2(inv.x, inv.y));
    const float2 hi = snake2(make_float2(x.z, x.w), make_float2(alpha.z, alpha.w), make_float2(inv.z, inv.w));
    return make_float4(lo.x, lo.y, hi.x, hi.y);
}

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

}  // namespace vxb
