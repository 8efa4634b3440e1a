// Fused residual unit for the narrow stages (C <= 128 channels):
//
//   y = x + pw(snake2(dw_d(snake1(x)))) + b   [-> next block's / final Snake]
//
// (reference residual_unit_forward_l2, src/audio-vae.cpp:1481-1518), one
// kernel instead of prologue + pointwise GEMM: x is read from HBM once per
// tile (the causal halo, 6*d rows, and the residual re-read come from L2)
// and y written once, 8 bytes per element instead of 16.
//
// Persistent CTAs over tiles of 128 tokens of one sequence.  The pointwise
// GEMM runs on the tensor cores with the tokens as M:
//   D[token][cout] = sum_k H[token][k] * W[cout][k]     (M = 128, N = C)
// A = H, the fp16 activation tile the CTA itself produced in shared memory
// (K-major, 128-byte swizzle); B = W, the unit's weights, dequantised (Q4_0)
// or copied (F16) into shared memory once per CTA; D in TMEM (two
// accumulators of C columns, so tile i's epilogue overlaps tile i+1's work).
//
// Warp roles (480 threads):
//   warp 9      slice loader: one TMA load per 32-channel slice of a tile, rows
//               [t0 - 6d, t0 + 128) of the sequence (rows before its start
//               read as zero: the causal padding), into a ring of slots that
//               runs several slices (and tiles) ahead of the producers.
//   warps 0-7   producers: per slice, snake1 in place, dilated causal k7
//               conv + bias + snake2 -> fp16 into the H tile.  A thread
//               computes the outputs q, q+d, q+2d, q+3d, whose 28 taps read
//               only 10 distinct rows.
//   warp 8      TMEM owner; lane 0 issues the MMAs (K steps of 16).
//   warp 14     residual loader: the boxes [128 tokens][32 channels] of x
//               that the epilogue adds, by TMA (128-byte swizzle) into a ring
//               that runs ahead of the epilogue.
//   warps 10-13 epilogue, one TMEM lane (= token) per thread, 32 channels at
//               a time: y = D + b + x is written back into the residual box
//               (swizzled, conflict-free per-row access; the fp16 variant as
//               dense 64-byte rows) and each warp sends its 32 rows out by
//               TMA, with no barrier across the epilogue warps.
// Every wait is bounded (the status word records a failure and the kernel
// returns); the CTA always frees its TMEM.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace vxb {

enum ResEpi : int {
    kResPlain = 0,     // y = x + pw + b (fp32)
    kResSnakeF16 = 1,  // y = snake(x + pw + b) (fp16: the next transposed conv's B operand)
    kResSnakeF32 = 2,  // y = snake(x + pw + b) (fp32: the final conv's input)
};

struct ResUnitArgs {
    const float* x;           // fp32 [B*T][C] residual stream
    void* y;                  // fp32 / fp16 [B*T][C]
    const float *a1, *i1;     // snake1 alpha, 1/(alpha + 1e-9) [C]
    const float* dw;          // depthwise taps [C][7]
    const float* db;          // depthwise bias [C]
    const float *a2, *i2;     // snake2 [C]
    const uint8_t* w;         // pointwise weight rows (row = cout): F16 [C][C] or Q4_0 (C/32 blocks of 18 B)
    int w_q4;                 // 1: Q4_0, 0: F16
    const float* pb;          // pointwise bias [C]
    const float *sa, *si;     // epilogue Snake (kResSnake*)
    int T, C, d;              // frames per sequence, channels, dilation
    int t_tiles, tiles;       // ceil(T / 128), batch * t_tiles
    int* status;
};

constexpr int kRuTT = 128;                 // tokens per tile (MMA M)
constexpr int kRuSlice = 32;               // channels per slice / residual box (one 128-byte row)
constexpr int kRuMaxRows = kRuTT + 6 * 9;  // slice rows for dilation <= 9
constexpr int kRuThreads = 480;
constexpr int kRuSlotBytes = kRuMaxRows * kRuSlice * 4;  // 182 rows x 128 B
constexpr int kRuBoxBytes = kRuTT * kRuSlice * 4;        // 128 rows x 128 B
constexpr int kRuNE = 3;                                 // residual boxes in flight (fused kernel)
constexpr int kRuMaxNE = 6;                              // HG: as many as shared memory holds, up to 6
constexpr int kRuNH = 2;                                 // H buffers
constexpr int kRuMaxSlots = 4;
constexpr int kRuBarBytes = 256;
constexpr int kRuSmemLimit = 227 * 1024;

// Shared-memory layout for C channels (W, H, E 1024-byte aligned):
//   W  KB k-blocks of [C rows][128 B]   H  2 x KB k-blocks of [128 rows][128 B]
//   E  ne residual boxes                P  per-channel parameters (12 C floats)
//   X  slots of [182 rows][128 B]
struct RuLayout {
    int kb, w_bytes, h_off, e_off, p_off, x_off, bar_off, slots, total;
    int ne;  // residual boxes in flight
    int nh;  // H buffers
};

// hg: the H tiles come from global memory (the pointwise-only variant), no
// parameters or slices.  nh: H buffers (2, or 1 for the pointwise-only units
// that ru_nh picks; a compile-time constant in the kernel).
__host__ __device__ inline RuLayout ru_layout(int C, bool hg = false, int nh = kRuNH) {
    RuLayout L;
    L.kb = (C + 63) / 64;
    L.w_bytes = L.kb * C * 128;
    L.h_off = L.w_bytes;
    L.nh = nh;
    L.e_off = L.h_off + nh * L.kb * kRuTT * 128;
    // HG: the residual ring is what keeps the loads ahead of the epilogue (one
    // box less in flight made the unit 40 % slower), so where the room left
    // holds kRuMaxNE boxes it takes them (96 channels, batch 256: 182 -> 162 us
    // per unit); otherwise, and in the fused kernel, 3.  The kernel takes the
    // count as a template argument (a run-time modulo on the ring index cost
    // the 192-channel and Snake-output units 2-5 %).
    L.ne = kRuNE;
    if (hg && (kRuSmemLimit - 1024 - kRuBarBytes - L.e_off) / kRuBoxBytes >= kRuMaxNE) L.ne = kRuMaxNE;
    L.p_off = L.e_off + L.ne * kRuBoxBytes;
    L.x_off = L.p_off + (hg ? 0 : (12 * C * 4 + 127) / 128 * 128);
    const int room = kRuSmemLimit - 1024 - kRuBarBytes - L.x_off;
    L.slots = hg ? 0 : room / kRuSlotBytes;
    if (L.slots > kRuMaxSlots) L.slots = kRuMaxSlots;
    L.bar_off = L.x_off + (L.slots > 0 ? L.slots : 0) * kRuSlotBytes;
    L.total = L.bar_off + kRuBarBytes + 1024;
    return L;
}

// H buffers of a unit.  A pointwise-only unit with the plain epilogue whose
// two H buffers leave no room for kRuMaxNE residual boxes (C > 128) keeps one:
// the loader refills it as soon as the tile's MMAs have read it, and the next
// MMAs also wait for the epilogue to drain an accumulator, which takes longer
// (192 channels, batch 256: 189 -> 163 us per unit).  The Snake epilogues keep
// two H buffers and 3 boxes there (measured 182 us against 190 with one).
inline int ru_nh(int C, bool hg, int epi) {
    return hg && epi == kResPlain && ru_layout(C, true).ne < kRuMaxNE ? 1 : kRuNH;
}

// Byte offset of (row, channel c < 32) in a residual box: rows of 128 B with
// the 128-byte swizzle (16-byte chunk index XOR row % 8), as TMA writes it.
__device__ __forceinline__ uint32_t ru_box_off(uint32_t row, uint32_t c) {
    return row * 128u + ((((c >> 2) ^ row) & 7u) << 4) + (c & 3u) * 4u;
}

// Producer-warp barrier (named barrier 1, 256 threads), OR-ing a predicate
// across the 256 producer threads (a uniform bail-out).
__device__ __forceinline__ bool ru_prod_bar_any(bool p) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n barrier.red.or.pred q, 1, 256, p;\n"
        " selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(p))
        : "memory");
    return r != 0;
}

// tcgen05.ld of 32 lanes x 16 columns without the wait (tmem_wait_ld completes it).
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// HG = true: the pointwise-only variant for stages whose fused form does not
// fit shared memory (C <= 192): the H tiles (the prologue kernel's fp16
// output [B*T][C]) arrive by TMA (tmap_h, boxes {64 k, 128 tokens}, 128-byte
// swizzle) into the H buffers, issued by the loader warp; the producer warps
// idle.  Everything else is the same kernel.
template <int EPI, bool HG, int NE, int NH>
__global__ void __launch_bounds__(kRuThreads, 1)
    resunit_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_res,
                   const __grid_constant__ CUtensorMap tmap_y, const __grid_constant__ CUtensorMap tmap_h,
                   const ResUnitArgs args) {
    const int C = args.C;
    static_assert(NE >= 1 && NE <= kRuMaxNE && NH >= 1 && NH <= kRuNH && (NH == kRuNH || HG), "rings");
    const RuLayout L = ru_layout(C, HG, NH);  // L.ne == NE (the host picks the instance)
    const int NS = L.slots;
    extern __shared__ uint8_t ru_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ru_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sW = smem;
    uint8_t* sH = smem + L.h_off;
    uint8_t* sE = smem + L.e_off;
    uint8_t* sX = smem + L.x_off;
    // parameters: taps [7][C] (tap-major: one float4 per tap and channel quad),
    // then snake1 alpha / inv, dw bias, snake2 alpha / inv, [C] each
    float* sP = reinterpret_cast<float*>(smem + L.p_off);
    float* sTap = sP;
    float* sA1 = sP + 7 * C;
    float* sI1 = sA1 + C;
    float* sDB = sI1 + C;
    float* sA2 = sDB + C;
    float* sI2 = sA2 + C;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);  // [NS] slice landed (TMA bytes)
    uint64_t* empty = full + kRuMaxSlots;                            // [NS] slice consumed (8 producer warps)
    uint64_t* efull = empty + kRuMaxSlots;                           // [ne] residual box landed
    uint64_t* eempty = efull + kRuMaxNE;                             // [ne] residual box released
    uint64_t* hfull = eempty + kRuMaxNE;                             // [NH] H written (8 producer warps)
    uint64_t* hempty = hfull + kRuNH;                                // [NH] H read by the MMAs
    uint64_t* afull = hempty + kRuNH;                                // [2] accumulator complete
    uint64_t* aempty = afull + 2;                                    // [2] accumulator drained (4 warps)
    uint64_t* done_bar = aempty + 2;                                 // all MMAs of the CTA complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nslices = C / kRuSlice;
    const int d = args.d, halo = 6 * d, R = kRuTT + halo;  // slot rows
    const int acc_cols = L.kb == 3 ? 256 : 64 * L.kb;  // accumulator stride: a power of two
    const uint32_t tmem_cols = 2 * acc_cols <= 128 ? 128 : (2 * acc_cols <= 256 ? 256 : 512);

    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 8);
        }
        for (int i = 0; i < NE; ++i) {
            mbar_init(&efull[i], 1);
            mbar_init(&eempty[i], 4);  // one arrival per epilogue warp
        }
        for (int i = 0; i < NH; ++i) {
            mbar_init(&hfull[i], HG ? 1 : 8);
            mbar_init(&hempty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&afull[i], 1);
            mbar_init(&aempty[i], 4);
        }
        mbar_init(done_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(HG ? &tmap_h : &tmap_x);
        prefetch_tmap(&tmap_res);
        prefetch_tmap(&tmap_y);
    }
    if (warp == 8) tmem_alloc(tmem_slot, tmem_cols);

    // W -> shared memory, K-major 128-byte swizzle: k-block kb holds rows
    // (cout) 0..C-1 x k in [64 kb, 64 kb + 64).  Weights are not written by
    // earlier kernels, so this overlaps the previous kernel (before the
    // grid dependency wait).  One item = 8 consecutive k of one row.
    {
        const int kchunks = C / 8;
        for (int item = threadIdx.x; item < C * kchunks; item += kRuThreads) {
            const int row = item / kchunks, kc = item - row * kchunks;
            const int k = kc * 8;
            uint4 v;
            if (args.w_q4) {
                // block k/32 of the row; k%32 < 16: low nibbles of bytes k%32..+7, else high nibbles of bytes k%32-16..+7
                const uint8_t* blk = args.w + (static_cast<size_t>(row) * (C / 32) + (k >> 5)) * 18;
                const int j0 = k & 15;
                const __half2 d2 = __half2half2(__ushort_as_half(static_cast<uint16_t>(blk[0] | (blk[1] << 8))));
                uint32_t q0 = 0, q1 = 0;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    q0 |= static_cast<uint32_t>(blk[2 + j0 + j]) << (8 * j);
                    q1 |= static_cast<uint32_t>(blk[2 + j0 + 4 + j]) << (8 * j);
                }
                v = q4_dequant8(q0, q1, (k & 31) >= 16, d2);
            } else {
                v = *reinterpret_cast<const uint4*>(args.w + (static_cast<size_t>(row) * C + k) * 2);
            }
            *reinterpret_cast<uint4*>(sW + (k >> 6) * (C * 128) + sw128_kmajor_off(row, k & 63)) = v;
        }
    }
    for (int i = threadIdx.x; i < (HG ? 0 : C); i += kRuThreads) {
#pragma unroll
        for (int k = 0; k < 7; ++k) sTap[k * C + i] = args.dw[i * 7 + k];
        sA1[i] = args.a1[i];
        sI1[i] = args.i1[i];
        sDB[i] = args.db[i];
        sA2[i] = args.a2[i];
        sI2[i] = args.i2[i];
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Only the warps that touch activations in global memory wait for the
    // previous kernel (the loaders, the epilogue's stores); the producers and
    // the MMA issuer work on shared memory and TMEM alone.
    if (warp >= 9) grid_dep_sync();

    if (warp == 9) {
        if (lane == 0) {
            // --------------------------------------------------- loader --
            if (HG) {
                int i = 0;
                for (int tile = blockIdx.x; tile < args.tiles && !*abort_flag; tile += gridDim.x, ++i) {
                    const int hbuf = i % NH;
                    const uint32_t hph = (i / NH) & 1;
                    if (!mbar_wait(&hempty[hbuf], hph ^ 1, abort_flag, args.status, kErrWaitEmpty)) break;
                    const int b = tile / args.t_tiles;
                    const int t0 = (tile - b * args.t_tiles) * kRuTT;
                    mbar_arrive_expect_tx(&hfull[hbuf], static_cast<uint32_t>(L.kb) * kRuTT * 128);
                    for (int kb = 0; kb < L.kb; ++kb)
                        tma_load_2d(sH + (hbuf * L.kb + kb) * (kRuTT * 128), &tmap_h, &hfull[hbuf], kb * 64,
                                    b * args.T + t0);
                }
            }
            const uint32_t tx = static_cast<uint32_t>(R) * kRuSlice * 4;
            int it = 0;
            for (int tile = blockIdx.x; tile < (HG ? 0 : args.tiles) && !*abort_flag; tile += gridDim.x) {
                const int b = tile / args.t_tiles;
                const int t0 = (tile - b * args.t_tiles) * kRuTT;
                bool ok = true;
                for (int s = 0; s < nslices; ++s, ++it) {
                    const int slot = it % NS;
                    if (!mbar_wait(&empty[slot], ((it / NS) & 1) ^ 1, abort_flag, args.status, kErrWaitEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[slot], tx);
                    tma_load_3d(sX + slot * kRuSlotBytes, &tmap_x, &full[slot], s * kRuSlice, t0 - halo, b);
                }
                if (!ok) break;
            }
            if (*abort_flag) {
                // failure path only: give copies already in flight time to land
                const unsigned long long t0 = globaltimer_ns();
                while (globaltimer_ns() - t0 < 1000000ull) {
                }
            }
        }
    } else if (warp == 14) {
        if (lane == 0) {
            // ----------------------------------------- residual loader --
            int g = 0;
            for (int tile = blockIdx.x; tile < args.tiles && !*abort_flag; tile += gridDim.x) {
                const int b = tile / args.t_tiles;
                const int t0 = (tile - b * args.t_tiles) * kRuTT;
                bool ok = true;
                for (int j = 0; j < nslices; ++j, ++g) {
                    const int e = g % NE;
                    if (!mbar_wait(&eempty[e], ((g / NE) & 1) ^ 1, abort_flag, args.status, kErrWaitEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&efull[e], kRuBoxBytes);
                    tma_load_3d(sE + e * kRuBoxBytes, &tmap_res, &efull[e], j * kRuSlice, t0, b);
                }
                if (!ok) break;
            }
            if (*abort_flag) {
                const unsigned long long t0 = globaltimer_ns();
                while (globaltimer_ns() - t0 < 1000000ull) {
                }
            }
        }
    } else if (warp < 8 && !HG) {
        // ------------------------------------------------------ producers --
        const int tid = threadIdx.x;   // 0..255
        const int cx = tid & 7;        // float4 column within the 32-channel slice
        const int ry = tid >> 3;       // row group 0..31
        // output sets {q0, q0+d, q0+2d, q0+3d}: blocks of 4d rows, d sets each;
        // this thread takes sets ry and ry + 32 (at most 36 sets for d <= 9)
        const int nsets = (kRuTT + 4 * d - 1) / (4 * d) * d;
        auto set_q0 = [&](int set) { return set < nsets ? (set / d) * 3 * d + set : kRuTT; };  // kRuTT: no set
        const int q0a = set_q0(ry), q0b = set_q0(ry + 32);
        int it = 0, i = 0;
        bool bail = false;
        for (int tile = blockIdx.x; tile < args.tiles && !bail; tile += gridDim.x, ++i) {
            const int hbuf = i & 1;
            bool ok = mbar_wait(&hempty[hbuf], ((i >> 1) & 1) ^ 1, abort_flag, args.status, kErrWaitEmpty);
            if (ru_prod_bar_any(!ok || *abort_flag != 0)) break;
            const int b = tile / args.t_tiles;
            const int t0 = (tile - b * args.t_tiles) * kRuTT;
            const int tv = args.T - t0;  // valid rows of the tile (may exceed 128)
            for (int s = 0; s < nslices; ++s, ++it) {
                const int slot = it % NS;
                float4* xs = reinterpret_cast<float4*>(sX + slot * kRuSlotBytes);
                ok = mbar_wait(&full[slot], (it / NS) & 1, abort_flag, args.status, kErrWaitFull);
                const int c = s * kRuSlice + cx * 4;
                if (ok) {
                    // all rows of this thread loaded, activated and stored in
                    // lockstep: independent chains for the scheduler
                    constexpr int kRows = (kRuMaxRows + 31) / 32;
                    const float4 al = *reinterpret_cast<const float4*>(sA1 + c);
                    const float4 iv = *reinterpret_cast<const float4*>(sI1 + c);
                    float4 v[kRows];
#pragma unroll
                    for (int m = 0; m < kRows; ++m) {
                        const int r = min(ry + 32 * m, R - 1);
                        v[m] = xs[r * 8 + cx];
                    }
#pragma unroll
                    for (int m = 0; m < kRows; ++m) v[m] = snake4(v[m], al, iv);
#pragma unroll
                    for (int m = 0; m < kRows; ++m)
                        if (ry + 32 * m < R) xs[(ry + 32 * m) * 8 + cx] = v[m];
                }
                if (ru_prod_bar_any(!ok)) {  // also orders snake1's writes before the taps read them
                    bail = true;
                    break;
                }
                float2 wlo[7], whi[7];
#pragma unroll
                for (int k = 0; k < 7; ++k) {
                    const float4 w4 = *reinterpret_cast<const float4*>(sTap + k * C + c);
                    wlo[k] = make_float2(w4.x, w4.y);
                    whi[k] = make_float2(w4.z, w4.w);
                }
                const float4 bb = *reinterpret_cast<const float4*>(sDB + c);
                const float4 al2 = *reinterpret_cast<const float4*>(sA2 + c);
                const float4 iv2 = *reinterpret_cast<const float4*>(sI2 + c);
                uint8_t* hk = sH + (hbuf * L.kb + (c >> 6)) * (kRuTT * 128);
                const int kin = c & 63;
#pragma unroll 1
                for (int e = 0; e < 2; ++e) {
                    const int q0 = e == 0 ? q0a : q0b;  // outputs q0 + j*d, j < 4
                    if (q0 >= kRuTT) break;
                    // rows q0 + m*d, m < 10 (output j uses m = j..j+6)
                    float4 u[10];
#pragma unroll
                    for (int m = 0; m < 10; ++m) {
                        const int rr = q0 + m * d;
                        u[m] = rr < R ? xs[rr * 8 + cx] : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                    // the four outputs in lockstep (no control flow until the stores)
                    float2 lo[4], hi[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        lo[j] = make_float2(bb.x, bb.y);
                        hi[j] = make_float2(bb.z, bb.w);
                    }
#pragma unroll
                    for (int k = 0; k < 7; ++k) {  // taps in order, one fma per tap and lane
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            lo[j] = ffma2(make_float2(u[j + k].x, u[j + k].y), wlo[k], lo[j]);
                            hi[j] = ffma2(make_float2(u[j + k].z, u[j + k].w), whi[k], hi[j]);
                        }
                    }
                    float4 yv[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) yv[j] = snake4(make_float4(lo[j].x, lo[j].y, hi[j].x, hi[j].y), al2, iv2);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int q = q0 + j * d;
                        if (q < kRuTT) {
                            const __half2 h01 = __floats2half2_rn(yv[j].x, yv[j].y);
                            const __half2 h23 = __floats2half2_rn(yv[j].z, yv[j].w);
                            uint2 pk;
                            pk.x = q < tv ? *reinterpret_cast<const uint32_t*>(&h01) : 0u;
                            pk.y = q < tv ? *reinterpret_cast<const uint32_t*>(&h23) : 0u;
                            *reinterpret_cast<uint2*>(hk + sw128_kmajor_off(q, kin)) = pk;
                        }
                    }
                }
                // generic-proxy writes (snake1 in the slot, H) before the slot
                // is refilled by TMA and before the MMAs read H
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
            if (bail) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&hfull[hbuf]);
        }
    } else if (warp == 8) {
        if (lane == 0) {
            // ------------------------------------------------- MMA issuer --
            const uint32_t idesc = make_idesc_f16(kRuTT, C, 0);
            int i = 0;
            for (int tile = blockIdx.x; tile < args.tiles; tile += gridDim.x, ++i) {
                const int acc = i & 1;
                const int hbuf = i % NH;
                const uint32_t hph = (i / NH) & 1;
                if (!mbar_wait(&aempty[acc], ((i >> 1) & 1) ^ 1, abort_flag, args.status, kErrWaitAccum)) break;
                if (!mbar_wait(&hfull[hbuf], hph, abort_flag, args.status, kErrWaitFull)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * acc_cols;
                const uint32_t h_addr = smem_u32(sH + hbuf * L.kb * (kRuTT * 128));
                const uint32_t w_addr = smem_u32(sW);
                for (int k16 = 0; k16 < C / 16; ++k16) {
                    const int kb = k16 >> 2, kk = k16 & 3;
                    const uint64_t adesc = make_sdesc(h_addr + kb * (kRuTT * 128) + kk * 32, 16, 1024);
                    const uint64_t bdesc = make_sdesc(w_addr + kb * (C * 128) + kk * 32, 16, 1024);
                    umma_f16(d_tmem, adesc, bdesc, idesc, k16 != 0);
                }
                umma_commit(&hempty[hbuf]);
                umma_commit(&afull[acc]);
            }
        }
    } else if (warp >= 10 && warp < 14) {
        // ------------------------------------------------------- epilogue --
        // Each warp owns the 32 rows (tokens) of its TMEM quadrant in every
        // residual box: it reads them, writes y back in place (fp16: as a
        // dense [32][64 B] block inside its own rows' bytes) and sends them
        // out with its own TMA store -- no barrier across the epilogue warps.
        // A box is released (eempty, 4 arrivals) once each warp's store of it
        // has read shared memory.
        const int q = warp & 3;                  // TMEM lane quadrant
        const int row = q * 32 + lane;           // token within the tile
        const int nbox = nslices;                // residual boxes per tile
        int g = 0, i = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < args.tiles && ok; tile += gridDim.x, ++i) {
            const int acc = i & 1;
            ok = mbar_wait(&afull[acc], (i >> 1) & 1, abort_flag, args.status, kErrWaitAccum);
            if (__any_sync(0xffffffffu, !ok)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int b = tile / args.t_tiles;
            const int t0 = (tile - b * args.t_tiles) * kRuTT;
            const uint32_t t_row = tmem_base + acc * acc_cols + (static_cast<uint32_t>(q * 32) << 16);
            for (int j = 0; j < nbox; ++j, ++g) {
                const int c0 = j * kRuSlice;
                uint32_t r[32];
                tmem_ld16_issue(t_row + c0, r);
                tmem_ld16_issue(t_row + c0 + 16, r + 16);
                tmem_wait_ld();
                if (j == nbox - 1) {
                    // accumulator fully read: the MMAs of tile i + 2 may reuse it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&aempty[acc]);
                }
                const bool landed = mbar_wait(&efull[g % NE], (g / NE) & 1, abort_flag, args.status,
                                              kErrWaitFull);
                if (__any_sync(0xffffffffu, !landed)) {
                    ok = false;
                    break;
                }
                uint8_t* box = sE + (g % NE) * kRuBoxBytes;
                uint8_t* own = box + q * 32 * 128;  // this warp's rows (4 KB, 1024-byte aligned)
                uint2 h16[8];
#pragma unroll
                for (int cq = 0; cq < 8; ++cq) {
                    const float4 pb = __ldg(reinterpret_cast<const float4*>(args.pb + c0) + cq);
                    float4* px = reinterpret_cast<float4*>(box + ru_box_off(row, cq * 4));
                    const float4 xr = *px;
                    float4 v;
                    v.x = (__uint_as_float(r[4 * cq + 0]) + pb.x) + xr.x;
                    v.y = (__uint_as_float(r[4 * cq + 1]) + pb.y) + xr.y;
                    v.z = (__uint_as_float(r[4 * cq + 2]) + pb.z) + xr.z;
                    v.w = (__uint_as_float(r[4 * cq + 3]) + pb.w) + xr.w;
                    if (EPI != kResPlain) {
                        const float4 sa = __ldg(reinterpret_cast<const float4*>(args.sa + c0) + cq);
                        const float4 si = __ldg(reinterpret_cast<const float4*>(args.si + c0) + cq);
                        v = snake4(v, sa, si);
                    }
                    if (EPI == kResSnakeF16) {
                        const __half2 h01 = __floats2half2_rn(v.x, v.y);
                        const __half2 h23 = __floats2half2_rn(v.z, v.w);
                        h16[cq].x = *reinterpret_cast<const uint32_t*>(&h01);
                        h16[cq].y = *reinterpret_cast<const uint32_t*>(&h23);
                    } else {
                        *px = v;
                    }
                }
                if (EPI == kResSnakeF16) {
                    __syncwarp();  // the warp's fp32 rows are read before the fp16 block overwrites them
#pragma unroll
                    for (int cq = 0; cq < 8; ++cq) *reinterpret_cast<uint2*>(own + lane * 64 + cq * 8) = h16[cq];
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    // the warp's store of box g - 1 has read its rows: release that box
                    bulk_wait_read<0>();
                    if (g > 0) mbar_arrive(&eempty[(g - 1) % NE]);
                    // rows past the sequence end fall outside the tensor and are not written
                    tma_store_3d(&tmap_y, own, c0, t0 + q * 32, b);
                    bulk_commit();
                }
            }
        }
        if (lane == 0) bulk_wait_all();  // stores done before the CTA's shared memory goes away
    }

    if (warp == 8 && lane == 0) {
        // every MMA this CTA issued has completed before TMEM is freed (also
        // on the failure paths, where no epilogue waited for the last ones)
        umma_commit(done_bar);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(done_bar, 0) && globaltimer_ns() - t0 < kWaitNs) {
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) tmem_dealloc(tmem_base, tmem_cols);
}

}  // namespace vxb
