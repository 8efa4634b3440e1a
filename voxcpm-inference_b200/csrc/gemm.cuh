// Implicit-GEMM convolution kernel on the 5th-generation tensor cores.
//
// One CTA computes a 128 x BN tile of D = A * B^T with tcgen05.mma
// (kind::f16, fp16 operands, fp32 accumulator in TMEM):
//   * A = conv weights (M = output rows, K = input channels), either fp16
//     through TMA or Q4_0 blocks dequantised to fp16 by producer warps inside
//     the mainloop; K-major for pointwise convs (the GGUF [Cin, Cout] layout,
//     rows = Cout) and MN-major for the transposed convs (the folded GGUF
//     [2s*Cout, Cin] layout, rows = Cin, j = cout*2s + k contiguous).
//   * B = activations, fp16 [N tokens][K channels] (K-major), through TMA.
// The epilogue reads the accumulator with tcgen05.ld and fuses bias, the
// residual add, the next layer's Snake (fp16 or fp32 output), or, for a
// transposed conv, the col2im overlap-add of the two taps that land on each
// output sample plus bias.
//
// Warp roles: warp 0 lane 0 issues TMA loads, warp 1 owns TMEM and lane 0
// issues the MMAs, warps 4-7 (Q4_0 variants only) dequantise A; warps 0-3
// then run the epilogue (warp w reads TMEM lanes 32w..32w+31).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace vxb {

enum AKind : int {
    kAF16K = 0,   // fp16, K-major, TMA box {64 k, 128 m}
    kAF16MN = 1,  // fp16, MN-major, two TMA boxes {64 m, 64 k}
    kAQ4K = 2,    // Q4_0 rows along K (pointwise [Cin, Cout]), dequantised in smem
    kAQ4MN = 3,   // Q4_0 rows along M (transposed conv [2s*Cout, Cin]), dequantised in smem
};

enum Epi : int {
    kEpiPW = 0,     // y[n][m] = acc + b[m] (+ r[n][m]) [-> snake]  -> fp32 or fp16
    kEpiConvT = 1,  // y[(n*s + r)][co] = D[co*2s + r][n] + D[co*2s + s + r][n-1] + b[co]
};

struct GemmArgs {
    int M, K, N;              // GEMM extents; M counts A rows of the whole layer
    const uint8_t* a_q4;      // Q4_0 blocks (kAQ4*), else unused
    int a_row_bytes;          // bytes per Q4_0 row
    const float* bias;        // [M] (PW) or [Cout] (ConvT)
    const float* res;         // fp32 [N][M] residual or null (PW)
    const float* snake_alpha; // [M] or null (PW)
    const float* snake_inv;   // [M] or null (PW)
    void* out;                // fp32 or fp16 [N][M] (PW); fp32 [N*s][Cout] (ConvT)
    int out_f16;              // PW: 1 = fp16 output
    int s, cout, cpt, seq_len;  // ConvT: stride, Cout, couts per tile, latent frames per sequence
    int* status;              // device status word (bounded-wait failures)
};

template <int BN>
struct GemmCfg {
    static constexpr int kBM = 128;
    static constexpr int kBK = 64;
    static constexpr int kABytes = kBM * kBK * 2;  // 16 KB
    static constexpr int kBBytes = BN * kBK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStages = BN >= 256 ? 4 : (BN >= 128 ? 5 : 6);
    static constexpr int kTmemCols = BN < 32 ? 32 : BN;
    static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA M=128 needs N % 16 == 0, 16..256");
};

template <int AK, int BN, int EPI>
__global__ void __launch_bounds__((AK >= kAQ4K) ? 256 : 128, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                const GemmArgs args) {
    using Cfg = GemmCfg<BN>;
    constexpr int S = Cfg::kStages;
    constexpr bool kQ4 = AK >= kAQ4K;
    constexpr bool kMN = (AK == kAF16MN) || (AK == kAQ4MN);
    constexpr int kNumDeqWarps = kQ4 ? 4 : 0;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
    uint64_t* empty_bar = full_bar + S;
    uint64_t* accum_bar = empty_bar + S;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_kb = (args.K + Cfg::kBK - 1) / Cfg::kBK;

    int m0, n_start;
    if (EPI == kEpiConvT) {
        m0 = blockIdx.x * (2 * args.s * args.cpt);
        n_start = blockIdx.y * (BN - 1) - 1;  // column 0 holds token n_first - 1
    } else {
        m0 = blockIdx.x * Cfg::kBM;
        n_start = blockIdx.y * BN;
    }

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full_bar[i], 1 + kNumDeqWarps);
            mbar_init(&empty_bar[i], 1);
        }
        mbar_init(accum_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&tmap_b);
        if (!kQ4) prefetch_tmap(&tmap_a);
    }
    if (warp == 1) tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // ------------------------------------------------------------ roles --
    if (warp == 0 && lane == 0) {
        // TMA producer: B always, A for the fp16 kinds.
        constexpr uint32_t kTx = kQ4 ? Cfg::kBBytes : Cfg::kStageBytes;
        for (int kb = 0; kb < num_kb; ++kb) {
            const int st = kb % S;
            if (!mbar_wait(&empty_bar[st], ((kb / S) & 1) ^ 1, abort_flag, args.status, kErrWaitEmpty)) break;
            uint8_t* a_dst = smem + st * Cfg::kStageBytes;
            uint8_t* b_dst = a_dst + Cfg::kABytes;
            mbar_arrive_expect_tx(&full_bar[st], kTx);
            const int k0 = kb * Cfg::kBK;
            if (AK == kAF16K) {
                tma_load_2d(a_dst, &tmap_a, &full_bar[st], k0, m0);
            } else if (AK == kAF16MN) {
                tma_load_2d(a_dst, &tmap_a, &full_bar[st], m0, k0);
                tma_load_2d(a_dst + 8192, &tmap_a, &full_bar[st], m0 + 64, k0);
            }
            tma_load_2d(b_dst, &tmap_b, &full_bar[st], k0, n_start);
        }
        if (*abort_flag) {
            // Failure path only: give copies already in flight time to land
            // before the CTA's shared memory goes away.
            const unsigned long long t0 = globaltimer_ns();
            while (globaltimer_ns() - t0 < 1000000ull) {
            }
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer.
        constexpr uint32_t idesc = make_idesc_f16(128, BN, kMN ? 1 : 0);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
            const int st = kb % S;
            if (!mbar_wait(&full_bar[st], (kb / S) & 1, abort_flag, args.status, kErrWaitFull)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t a_addr = smem_u32(smem + st * Cfg::kStageBytes);
            const uint32_t b_addr = a_addr + Cfg::kABytes;
#pragma unroll
            for (int kk = 0; kk < Cfg::kBK / 16; ++kk) {
                // K-major SW128: +32 B per 16 k inside the 128-B row.
                // MN-major SW128: +2 KB per 16 k (two 8-row k groups of 1 KB);
                // the two 64-element m halves are 8 KB apart (LBO).
                const uint64_t adesc = kMN ? make_sdesc(a_addr + kk * 2048, 8192, 1024)
                                           : make_sdesc(a_addr + kk * 32, 16, 1024);
                const uint64_t bdesc = make_sdesc(b_addr + kk * 32, 16, 1024);
                umma_f16(tmem_base, adesc, bdesc, idesc, (kb | kk) != 0);
            }
            umma_commit(&empty_bar[st]);
        }
        // Always publish: the accumulator barrier completes once every MMA
        // issued so far has finished, so TMEM is idle before it is freed even
        // on the failure path (the epilogue then sees the abort flag).
        (void)ok;
        umma_commit(accum_bar);
    } else if (kQ4 && warp >= 4) {
        // Q4_0 dequantisers: 128 threads fill the A tile of each stage.
        const int t = threadIdx.x - 128;
        for (int kb = 0; kb < num_kb; ++kb) {
            const int st = kb % S;
            if (!mbar_wait(&empty_bar[st], ((kb / S) & 1) ^ 1, abort_flag, args.status, kErrWaitEmpty)) break;
            uint8_t* a_dst = smem + st * Cfg::kStageBytes;
            const int k0 = kb * Cfg::kBK;
            if (AK == kAQ4K) {
                // thread t -> row m0 + t, two 32-element blocks along k; all
                // loads of both blocks are issued before any is used.
                const int m = m0 + t;
                uint32_t q4[2][4];
                float dd[2];
#pragma unroll
                for (int hb = 0; hb < 2; ++hb) {
                    const int kx = k0 + hb * 32;
                    dd[hb] = 0.f;
                    q4[hb][0] = q4[hb][1] = q4[hb][2] = q4[hb][3] = 0u;
                    if (m < args.M && kx < args.K) {
                        const uint16_t* b16 = reinterpret_cast<const uint16_t*>(
                            args.a_q4 + static_cast<size_t>(m) * args.a_row_bytes + (kx >> 5) * 18);
                        dd[hb] = half_bits_to_float(__ldg(b16));
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            q4[hb][j] = static_cast<uint32_t>(__ldg(b16 + 1 + 2 * j)) |
                                        (static_cast<uint32_t>(__ldg(b16 + 2 + 2 * j)) << 16);
                    }
                }
#pragma unroll
                for (int hb = 0; hb < 2; ++hb) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        __align__(16) __half v[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const int j = (c & 1) * 8 + e;
                            const uint32_t byte = (q4[hb][j >> 2] >> ((j & 3) * 8)) & 0xFFu;
                            const uint32_t nib = c < 2 ? (byte & 15u) : (byte >> 4);
                            v[e] = __float2half_rn(static_cast<float>(static_cast<int>(nib) - 8) * dd[hb]);
                        }
                        *reinterpret_cast<uint4*>(a_dst + sw128_kmajor_off(t, hb * 32 + c * 8)) =
                            *reinterpret_cast<const uint4*>(v);
                    }
                }
            } else {
                // Work item = one Q4_0 block (32 consecutive m at one k row)
                // that intersects the tile's m range [m0, m0 + 128).  m0 is a
                // multiple of 8, so a block lands on four aligned 16-byte
                // chunks of the MN-major swizzled tile.
                const int b_first = m0 >> 5;
                const int nblk = ((m0 + 127) >> 5) - b_first + 1;  // <= 5
                const int items = 64 * nblk;
#pragma unroll
                for (int it = 0; it < 3; ++it) {
                    const int item = t + it * 128;
                    if (item >= items) break;
                    const int kl = item / nblk;
                    const int blk = b_first + item % nblk;
                    const int k = k0 + kl;
                    uint32_t q4[4] = {0u, 0u, 0u, 0u};  // 16 nibble bytes
                    float d = 0.f;
                    const bool valid = k < args.K && blk * 32 < args.M;
                    if (valid) {
                        const uint16_t* b16 = reinterpret_cast<const uint16_t*>(
                            args.a_q4 + static_cast<size_t>(k) * args.a_row_bytes + static_cast<size_t>(blk) * 18);
                        d = half_bits_to_float(__ldg(b16));
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            q4[j] = static_cast<uint32_t>(__ldg(b16 + 1 + 2 * j)) |
                                    (static_cast<uint32_t>(__ldg(b16 + 2 + 2 * j)) << 16);
                    }
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        // elements 8c..8c+7 of the block: low nibbles for c < 2
                        const int ml = blk * 32 + c * 8 - m0;
                        if (ml < 0 || ml >= 128) continue;
                        __align__(16) __half v[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const int j = (c & 1) * 8 + e;  // byte index 0..15
                            const uint32_t byte = (q4[j >> 2] >> ((j & 3) * 8)) & 0xFFu;
                            const uint32_t nib = c < 2 ? (byte & 15u) : (byte >> 4);
                            v[e] = __float2half_rn(static_cast<float>(static_cast<int>(nib) - 8) * d);
                        }
                        const int h = ml >> 6, mc = (ml & 63) >> 3;
                        const uint32_t off = h * 8192 + (kl >> 3) * 1024 + (kl & 7) * 128 + (((mc ^ kl) & 7) << 4);
                        *reinterpret_cast<uint4*>(a_dst + off) = *reinterpret_cast<const uint4*>(v);
                    }
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full_bar[st]);
        }
    }

    // ----------------------------------------------------------- epilogue --
    if (warp < 4) {
        __syncwarp();
        bool ok = mbar_wait(accum_bar, 0, abort_flag, args.status, kErrWaitAccum);
        ok = __all_sync(0xffffffffu, ok && *abort_flag == 0);  // tcgen05.ld needs a uniform warp
        tc_fence_after();
        const int row = warp * 32 + lane;  // D row == TMEM lane
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
        if (EPI == kEpiPW) {
            const int m = m0 + row;
            const bool mv = ok && m < args.M;
            const float b = mv ? args.bias[m] : 0.f;
            const float al = (mv && args.snake_alpha) ? args.snake_alpha[m] : 0.f;
            const float iv = (mv && args.snake_alpha)
                                 ? (args.snake_inv ? args.snake_inv[m] : 1.0f / (al + 1e-9f))
                                 : 0.f;
            const float* __restrict__ res = args.res;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                float v[16];
                if (ok) tmem_ld16(t_row + c0, v);  // .sync.aligned: whole warp
                const int nb = n_start + c0;
                if (!mv || nb >= args.N) continue;
                const int cnt = min(16, args.N - nb);
                float r[16];
#pragma unroll
                for (int i = 0; i < 16; ++i)  // issue every residual load first
                    r[i] = (res && i < cnt) ? __ldg(res + static_cast<size_t>(nb + i) * args.M + m) : 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    if (i >= cnt) break;
                    const size_t o = static_cast<size_t>(nb + i) * args.M + m;
                    float y = v[i] + b + r[i];
                    if (args.snake_alpha) y = snake(y, al, iv);
                    if (args.out_f16) {
                        static_cast<__half*>(args.out)[o] = __float2half_rn(y);
                    } else {
                        static_cast<float*>(args.out)[o] = y;
                    }
                }
            }
        } else {
            // ConvT: stage D (fp32) in the now idle pipeline smem, then
            // overlap-add the two taps of every output sample.
            constexpr int LD = BN + 1;
            float* sD = reinterpret_cast<float*>(smem);
            if (ok) {
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 16) {
                    float v[16];
                    tmem_ld16(t_row + c0, v);
#pragma unroll
                    for (int i = 0; i < 16; ++i) sD[row * LD + c0 + i] = v[i];
                }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (ok) {
                const int s = args.s;
                const int co_lo = blockIdx.x * args.cpt;
                const int cpt = min(args.cpt, args.cout - co_lo);
                const int n_first = n_start + 1;
                const int n_tok = min(BN - 1, args.N - n_first);
                const int total = n_tok * s * cpt;
                float* out = static_cast<float*>(args.out);
                for (int idx = threadIdx.x; idx < total; idx += 128) {
                    const int co_l = idx % cpt;
                    const int rest = idx / cpt;
                    const int r = rest % s;
                    const int nn = rest / s;
                    const int n = n_first + nn;
                    float y = sD[(co_l * 2 * s + r) * LD + nn + 1] + args.bias[co_lo + co_l];
                    if (n % args.seq_len != 0) y += sD[(co_l * 2 * s + s + r) * LD + nn];
                    out[(static_cast<size_t>(n) * s + r) * args.cout + co_lo + co_l] = y;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace vxb
