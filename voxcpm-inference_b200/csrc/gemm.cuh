// Implicit-GEMM convolution kernel on the 5th-generation tensor cores.
//
// Persistent, warp-specialised: each CTA walks tiles blockIdx.x,
// blockIdx.x + gridDim.x, ... of D = A * B^T (128 x BN tiles, K steps of 64)
// with tcgen05.mma (kind::f16: fp16 operands, fp32 accumulator in TMEM):
//   * A = conv weights (M = output rows, K = input channels), either fp16
//     through TMA or Q4_0 blocks whose raw bytes arrive by TMA and are
//     dequantised to fp16 in shared memory inside the mainloop; K-major for
//     pointwise convs (the GGUF [Cin, Cout] layout, rows = Cout) and MN-major
//     for the transposed convs (the folded GGUF [2s*Cout, Cin] layout,
//     rows = Cin, j = cout*2s + k contiguous).
//   * B = activations, fp16 [N tokens][K channels] (K-major), through TMA.
// Two TMEM accumulators let the epilogue of tile i overlap the mainloop of
// tile i+1.  The epilogue fuses bias, the residual add, the next layer's
// Snake (fp16 or fp32 output), or, for a transposed conv, the col2im
// overlap-add of the two taps that land on each output sample plus bias.
//
// Warp roles: warp 0 lane 0 issues TMA loads, warp 1 owns TMEM and lane 0
// issues the MMAs, warps 4-7 and 8-11 are two epilogue warpgroups (group g
// drains accumulator g, i.e. every other tile; warp w reads TMEM lanes
// 32*(w%4)...), warps 12-15 (Q4_0 variants) dequantise A.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace vxb {

enum AKind : int {
    kAF16K = 0,   // fp16, K-major, TMA box {64 k, 128 m}
    kAF16MN = 1,  // fp16, MN-major, two TMA boxes {64 m, 64 k}
    kAQ4K = 2,    // Q4_0 rows along K (pointwise [Cin, Cout]), raw bytes by TMA, dequantised in smem
    kAQ4MN = 3,   // Q4_0 rows along M (transposed conv [2s*Cout, Cin]), raw bytes by TMA, dequantised in smem
};

enum Epi : int {
    kEpiPW = 0,     // y[n][m] = acc + b[m] (+ r[n][m]) [-> snake]  -> fp32 or fp16
    kEpiConvT = 1,  // y[(n*s + r)][co] = D[co*2s + r][n] + D[co*2s + s + r][n-1] + b[co]
    kEpiPW32 = 2,   // as kEpiPW with fp32 output only (resident-A kernels): no fp16 staging
                    // buffers, their room spent on a residual ring twice as deep
};

struct GemmArgs {
    int M, K, N;              // GEMM extents; M counts A rows of the whole layer
    int m_tiles, n_tiles;     // tile grid (tile t -> m = t % m_tiles, n = t / m_tiles)
    const float* bias;        // [M] (PW) or [Cout] (ConvT)
    const float* res;         // fp32 [N][M] residual or null (PW)
    const float* snake_alpha; // [M] or null (PW)
    const float* snake_inv;   // [M] or null (PW)
    void* out;                // fp32 or fp16 [N][M] (PW); fp32 [N*s][Cout] (ConvT)
    int out_f16;              // PW: 1 = fp16 output
    int s, cout, cpt, seq_len;  // ConvT: stride, Cout, couts per tile, frames per sequence
    int skip;                 // ConvT: leading input frames per sequence whose outputs are not written
                              // (a streaming window's history row); output rows shift down by skip*s
    int v8;                   // ConvT: cpt == 8, Cout % 8 == 0, output 32-byte aligned: one 32-byte
                              // store per output row (both cout quads of a row on one thread)
    int* status;              // device status word (bounded-wait failures)
};

// Q4_0 weights are staged per k step from their split form (made by
// q4_split_kernel): nibbles [rows][blocks][16 B], each block's 32 values as
// four words of 8 in the q4_slot order, and the fp16 scales transposed,
// [blocks][rows], so that consecutive rows' scales are consecutive halves:
//   K-major (pointwise): 128 rows x 2 blocks -> nibbles 128 x 32 B, scales
//     2 block rows x 128 (box {128, 2});
//   MN-major (transposed conv): 64 k rows x the up to 5 blocks covering a
//     128-wide m range -> nibbles 64 x 80 B, scales 5 block rows x 64 k
//     (box {64, 5}).
constexpr int kQ4KNibBox = 32;     // bytes
constexpr int kQ4KScaleRows = 2;   // block rows of the scale box
constexpr int kQ4MNNibBox = 80;    // bytes
constexpr int kQ4MNScaleRows = 5;  // block rows of the scale box
constexpr int kQ4KScaleOff = 128 * kQ4KNibBox;   // scale area within the raw stage area
constexpr int kQ4MNScaleOff = 64 * kQ4MNNibBox;
constexpr int kQ4KRawBytes = kQ4KScaleOff + kQ4KScaleRows * 128 * 2;
constexpr int kQ4MNRawBytes = kQ4MNScaleOff + kQ4MNScaleRows * 64 * 2;

// Pointwise epilogue chunk: tokens per residual load / output store.  The
// host builds the residual and output tensor maps with boxes of
// {128 channels, kEpiChunk tokens}.
constexpr int kEpiChunk = 16;
constexpr int kBarrierBytes = 512;  // mbarriers + TMEM slot + abort flag

// RESKB > 0 (Q4_0 only): "resident A" -- every CTA keeps one m tile (the
// grid is a multiple of m_tiles) and dequantises that tile's whole weight
// column (K <= 64 * RESKB) once, into RESKB k blocks kept in shared memory
// for all its n tiles; the stages then carry only B tiles (and, for the
// first tile, the raw Q4_0 blocks).
template <int BN, bool Q4, int EPI, int RESKB = 0>
struct GemmCfg {
    static constexpr int kBM = 128;
    static constexpr int kBK = 64;
    static constexpr int kABytes = kBM * kBK * 2;  // 16 KB
    static constexpr int kBBytes = BN * kBK * 2;
    // >= max(kQ4KRawBytes, kQ4MNRawBytes), 1 KB granular; kEpiPW32 (K-major only): >= kQ4KRawBytes
    static constexpr int kRawBytes = Q4 ? (EPI == kEpiPW32 ? 5120 : 6144) : 0;
    static constexpr int kResABytes = RESKB * kABytes;
    static constexpr int kBOff = RESKB ? 0 : kABytes;            // B tile within a stage
    static constexpr int kStageBytes = kBOff + kBBytes + kRawBytes;
    static constexpr int kEpiLD = 36;                            // ConvT: row stride (carry at 3, columns at 4..35)
    static constexpr int kChunk = kEpiChunk;                     // PW: tokens per residual/output chunk
    static constexpr int kResBytes = kChunk * 128 * 4;           // PW: fp32 [16 tokens][128 channels]
    static constexpr int kOut16Bytes = kChunk * 128 * 2;         // PW: fp16 [16 tokens][128 channels]
    // PW: residual / output chunk buffers per group; loads run kEpiAhead
    // chunks ahead.  Narrow tiles (one or two tiles per CTA on short
    // sequences) take a ring of 2 and spend the room on mainloop stages.
    // kEpiPW32 keeps a ring of 4 with the resident A (2 chunks ahead: the
    // residual loads were the epilogue's wait at a ring of 2).
    static constexpr int kEpiRing = EPI == kEpiPW32 ? 4 : ((BN <= 64 || RESKB) ? 2 : 4);
    static constexpr int kEpiAhead = kEpiRing / 2;
    static constexpr int kGroupEpiBytes =
        EPI == kEpiConvT ? 128 * kEpiLD * 4 : kEpiRing * kResBytes + (EPI == kEpiPW ? kEpiRing * kOut16Bytes : 0);
    static constexpr int kEpiBytes = 2 * kGroupEpiBytes;         // two epilogue warpgroups
    static constexpr int kBudget =
        (EPI == kEpiPW32 ? 227 : 220) * 1024 - kEpiBytes - 1024 - kBarrierBytes - kResABytes;
    static constexpr int kStagesFit = kBudget / kStageBytes;
    static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
    static constexpr int kTmemCols = 2 * (BN < 32 ? 32 : BN);   // two accumulators
    static constexpr int kAccStride = BN < 32 ? 32 : BN;
    static constexpr int kSmemBytes = kResABytes + kStages * kStageBytes + kEpiBytes + 1024 + kBarrierBytes;
    static_assert(RESKB == 0 || Q4, "resident A is for Q4_0 weights");
    static_assert(EPI != kEpiPW32 || !Q4 || kRawBytes >= kQ4KRawBytes, "fp32-output kernel: Q4_0 K-major raw blocks");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
    static_assert((4 * kStages + 12) * 8 + 8 <= kBarrierBytes, "barrier area too small");
    static constexpr int kDqWarps = 4;                           // Q4_0: dequantiser warps (one per SM sub-partition)
    static constexpr int kThreads = Q4 ? 384 + 32 * kDqWarps : 384;
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA M=128 needs N % 16 == 0, 16..256");
    static_assert(kStages >= 2, "pipeline needs two stages");
};

template <int AK, int BN, int EPI, int RESKB = 0>
__global__ void __launch_bounds__((AK >= kAQ4K) ? 384 + 32 * GemmCfg<BN, true, EPI>::kDqWarps : 384, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                const __grid_constant__ CUtensorMap tmap_res, const __grid_constant__ CUtensorMap tmap_out,
                const __grid_constant__ CUtensorMap tmap_scale, const GemmArgs args) {
    constexpr bool kQ4 = AK >= kAQ4K;
    constexpr bool kMN = (AK == kAF16MN) || (AK == kAQ4MN);
    constexpr bool kRes = RESKB > 0;
    using Cfg = GemmCfg<BN, kQ4, EPI, RESKB>;
    static_assert(EPI == kEpiConvT || (BN >= 32 && BN <= 128), "pointwise tiles are 32..128 tokens wide");
    constexpr bool kPW = EPI != kEpiConvT;  // kEpiPW or kEpiPW32
    constexpr int S = Cfg::kStages;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* resA = smem;                          // kRes: the CTA's weight column, RESKB k blocks
    uint8_t* stages = smem + Cfg::kResABytes;
    float* sE = reinterpret_cast<float*>(stages + S * Cfg::kStageBytes);
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(stages + S * Cfg::kStageBytes + Cfg::kEpiBytes);
    uint64_t* ready_bar = full_bar + S;   // A tile dequantised (Q4 only)
    uint64_t* empty_bar = ready_bar + S;  // stage consumed by the MMAs
    uint64_t* tfull_bar = empty_bar + S;  // accumulator [2] complete
    uint64_t* tempty_bar = tfull_bar + 2; // accumulator [2] drained
    uint64_t* res_bar = tempty_bar + 2;   // PW residual chunk [group][4] landed
    uint64_t* raw_bar = res_bar + 8;      // Q4_0 raw blocks of a stage landed (the B tile lands on full_bar)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(raw_bar + S);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_kb = (args.K + Cfg::kBK - 1) / Cfg::kBK;
    const int num_tiles = args.m_tiles * args.n_tiles;
    const int rows_per_tile = EPI == kEpiConvT ? 2 * args.s * args.cpt : Cfg::kBM;
    // at most one tile per CTA: the epilogue warpgroups help dequantise (Q4_0)
    const bool dq_help = kQ4 && num_tiles <= static_cast<int>(gridDim.x);
    const int dq_threads = 32 * Cfg::kDqWarps + (dq_help ? 256 : 0);

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&ready_bar[i], dq_threads / 32);
            mbar_init(&empty_bar[i], 1);
            mbar_init(&raw_bar[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull_bar[i], 1);
            mbar_init(&tempty_bar[i], 4);
            for (int j = 0; j < 4; ++j) mbar_init(&res_bar[4 * i + j], 1);
        }
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&tmap_b);
        prefetch_tmap(&tmap_a);
        if (kQ4) prefetch_tmap(&tmap_scale);
        if (kPW) {
            prefetch_tmap(&tmap_out);
            if (args.res) prefetch_tmap(&tmap_res);
        }
    }
    if (warp == 1) tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // Stage st's weight (A) part for k step kb of the tile at row m0: fp16
    // tiles complete full_bar[st] (which also expects the B tile); Q4_0 raw
    // blocks complete raw_bar[st], so the dequantisers start as soon as they
    // land, and full_bar[st] then expects the B tile only.
    constexpr uint32_t kTx = (kQ4 ? 0 : Cfg::kABytes) + Cfg::kBBytes;
    auto issue_a = [&](int st, int kb, int m0) {
        uint8_t* a_dst = stages + st * Cfg::kStageBytes;
        uint8_t* r_dst = a_dst + Cfg::kBOff + Cfg::kBBytes;
        const int k0 = kb * Cfg::kBK;
        if (AK == kAQ4K) {
            mbar_arrive_expect_tx(&raw_bar[st], kQ4KRawBytes);
            tma_load_2d(r_dst, &tmap_a, &raw_bar[st], kb * kQ4KNibBox, m0);
            tma_load_2d(r_dst + kQ4KScaleOff, &tmap_scale, &raw_bar[st], m0, 2 * kb);
        } else if (AK == kAQ4MN) {
            mbar_arrive_expect_tx(&raw_bar[st], kQ4MNRawBytes);
            tma_load_2d(r_dst, &tmap_a, &raw_bar[st], (m0 >> 5) * 16, k0);
            tma_load_2d(r_dst + kQ4MNScaleOff, &tmap_scale, &raw_bar[st], k0, m0 >> 5);
        }
        mbar_arrive_expect_tx(&full_bar[st], kTx);
        if (AK == kAF16K) {
            tma_load_2d(a_dst, &tmap_a, &full_bar[st], k0, m0);
        } else if (AK == kAF16MN) {
            tma_load_2d(a_dst, &tmap_a, &full_bar[st], m0, k0);
            tma_load_2d(a_dst + 8192, &tmap_a, &full_bar[st], m0 + 64, k0);
        }
    };
    // The weights are not written by earlier kernels: the A parts of the
    // first min(S, num_kb) k steps of the CTA's first tile are issued before
    // the grid dependency wait (every stage is free at this point), so their
    // HBM latency overlaps the previous kernel.  Only the threads that touch
    // activations wait -- the producer (B tiles) and the epilogue (residual
    // in, output out); the MMA issuer and the dequantisers work on shared
    // memory and TMEM alone and start on the prefetched stages at once.
    // The tile's later k steps (beyond the S stages) are prefetched into L2.
    const int n_pre = blockIdx.x < num_tiles ? min(S, num_kb) : 0;
    if (warp == 0 && lane == 0 && n_pre > 0) {
        const int m0 = (blockIdx.x % args.m_tiles) * rows_per_tile;
        for (int kb = 0; kb < n_pre; ++kb) issue_a(kb, kb, m0);
        for (int kb = n_pre; kb < num_kb; ++kb) {
            const int k0 = kb * Cfg::kBK;
            if (AK == kAQ4K) {
                tma_prefetch_2d(&tmap_a, kb * kQ4KNibBox, m0);
                tma_prefetch_2d(&tmap_scale, m0, 2 * kb);
            } else if (AK == kAQ4MN) {
                tma_prefetch_2d(&tmap_a, (m0 >> 5) * 16, k0);
                tma_prefetch_2d(&tmap_scale, k0, m0 >> 5);
            } else if (AK == kAF16K) {
                tma_prefetch_2d(&tmap_a, k0, m0);
            } else {
                tma_prefetch_2d(&tmap_a, m0, k0);
                tma_prefetch_2d(&tmap_a, m0 + 64, k0);
            }
        }
    }
    if (warp >= 4 && warp < 12 && lane == 0) {
        // the epilogue's per-row parameters of the group's first tile into L2
        const int tile = blockIdx.x + ((warp - 4) >> 2) * gridDim.x;
        if (tile < num_tiles) {
            const int mt = tile % args.m_tiles, qq = warp & 3;
            if (kPW) {
                const int m = mt * Cfg::kBM + qq * 32;
                if (m < args.M) {
                    prefetch_l2(args.bias + m);
                    if (args.snake_alpha) prefetch_l2(args.snake_alpha + m);
                    if (args.snake_inv) prefetch_l2(args.snake_inv + m);
                }
            } else if (mt * args.cpt + qq * 32 < args.cout) {
                prefetch_l2(args.bias + mt * args.cpt + qq * 32);
            }
        }
    }
    if (warp == 0 || (warp >= 4 && warp < 12)) grid_dep_sync();

    // ------------------------------------------- Q4_0 dequantisers ------
    // Thread t of nthr dequantisers.  The dedicated warps (12..) always run
    // it; when every CTA has at most one tile (short GEMMs: streaming
    // steps), the epilogue warpgroups, idle until that tile's accumulator is
    // complete, run it too, tripling the dequantisation rate of the CTA's
    // only mainloop.
    constexpr int kDqThreads = 32 * Cfg::kDqWarps;
    auto dequant = [&](const int t, const int nthr) {
        // MN-major: item i -> k row kl = i % 64 and block bi = i / 64 of the
        // up to five that intersect [m0, m0 + 128); m0 is a multiple of 8, so
        // a block lands on four aligned 16-byte chunks of the MN-major tile.
        // The smem offsets of a thread's items depend on the tile only: they
        // are computed once per tile, not per k step.
        constexpr int kMnItems = (64 * 5 + kDqThreads - 1) / kDqThreads;
        constexpr uint32_t kNone = 0xFFFFFFFFu;
        uint32_t mn_src[kMnItems], mn_dst[kMnItems][4];
        int mn_kl[kMnItems], mn_bi[kMnItems];
        bool mn_mv[kMnItems];
        int it = 0, m0_prev = -1;
        for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
            if (kRes && tile != static_cast<int>(blockIdx.x)) break;  // the resident column is done
            const int m0 = (tile % args.m_tiles) * rows_per_tile;
            if (AK == kAQ4MN && m0 != m0_prev) {
                m0_prev = m0;
                const int b_first = m0 >> 5;
                const int nblk = ((m0 + 127) >> 5) - b_first + 1;
#pragma unroll
                for (int j = 0; j < kMnItems; ++j) {
                    const int i = t + j * nthr;
                    const int kl = i & 63, bi = i >> 6;
                    const int blk = b_first + bi;
                    mn_kl[j] = kl;
                    mn_bi[j] = bi;  // block row of the scale box
                    mn_mv[j] = blk * 32 < args.M;
                    mn_src[j] = bi < nblk ? static_cast<uint32_t>(kl * kQ4MNNibBox + bi * 16) : kNone;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {  // word c: elements 8c..8c+7 of the block
                        const int ml = blk * 32 + c * 8 - m0;
                        const int hh = ml >> 6, mc = (ml & 63) >> 3;
                        mn_dst[j][c] = (bi < nblk && ml >= 0 && ml < 128)
                                           ? static_cast<uint32_t>(hh * 8192 + (kl >> 3) * 1024 + (kl & 7) * 128 +
                                                                   (((mc ^ kl) & 7) << 4))
                                           : kNone;
                    }
                }
            }
            bool ok = true;
            for (int kb = 0; kb < num_kb; ++kb, ++it) {
                const int st = it % S;
                if (!mbar_wait(&raw_bar[st], (it / S) & 1, abort_flag, args.status, kErrWaitFull)) {
                    ok = false;
                    break;
                }
                uint8_t* a_dst = kRes ? resA + kb * Cfg::kABytes : stages + st * Cfg::kStageBytes;
                const uint8_t* raw = stages + st * Cfg::kStageBytes + Cfg::kBOff + Cfg::kBBytes;
                const int k0 = kb * Cfg::kBK;
                if (AK == kAQ4K) {
                    // item i -> row m0 + (i & 127), block hb = i >> 7 of the
                    // step's two (k0..k0+63): nibbles 16 B, the scale in
                    // block row hb of the box
#pragma unroll
                    for (int i = t; i < 256; i += nthr) {
                        const int r = i & 127, hb = i >> 7;
                        const int m = m0 + r;
                        const bool valid = m < args.M && k0 + hb * 32 < args.K;
                        const __half* sc = reinterpret_cast<const __half*>(raw + kQ4KScaleOff);
                        const __half2 d2 = __half2half2(valid ? sc[hb * 128 + r] : __float2half_rn(0.f));
                        const uint4 q = reinterpret_cast<const uint4*>(raw + r * kQ4KNibBox)[hb];
                        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                        for (int c = 0; c < 4; ++c)  // word c: elements 8c..8c+7 of the block
                            *reinterpret_cast<uint4*>(a_dst + sw128_kmajor_off(r, hb * 32 + c * 8)) =
                                q4_dequant8_split(qw[c], d2);
                    }
                } else {
                    const __half* sc = reinterpret_cast<const __half*>(raw + kQ4MNScaleOff);
#pragma unroll
                    for (int j = 0; j < kMnItems; ++j) {
                        if (mn_src[j] == kNone) continue;
                        const int kl = mn_kl[j];
                        const bool valid = mn_mv[j] && k0 + kl < args.K;
                        const __half2 d2 = __half2half2(valid ? sc[mn_bi[j] * 64 + kl] : __float2half_rn(0.f));
                        const uint4 q = *reinterpret_cast<const uint4*>(raw + mn_src[j]);
                        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            if (mn_dst[j][c] != kNone)
                                *reinterpret_cast<uint4*>(a_dst + mn_dst[j][c]) = q4_dequant8_split(qw[c], d2);
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ready_bar[st]);
            }
            if (!ok) break;
        }
    };
    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ TMA producer --
            int it = 0;
            for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
                const int m0 = (tile % args.m_tiles) * rows_per_tile;
                const int nt = tile / args.m_tiles;
                const int n_start = EPI == kEpiConvT ? nt * (BN - 1) - 1 : nt * BN;
                for (int kb = 0; kb < num_kb; ++kb, ++it) {
                    const int st = it % S;
                    if (it >= n_pre) {  // (the first n_pre A parts went out before the wait)
                        if (!mbar_wait(&empty_bar[st], ((it / S) & 1) ^ 1, abort_flag, args.status, kErrWaitEmpty))
                            break;
                        if (!kRes || it < num_kb) {
                            issue_a(st, kb, m0);
                        } else {
                            mbar_arrive_expect_tx(&full_bar[st], kTx);  // B only: A is resident
                        }
                    }
                    tma_load_2d(stages + st * Cfg::kStageBytes + Cfg::kBOff, &tmap_b, &full_bar[st],
                                kb * Cfg::kBK, n_start);
                }
            }
            if (*abort_flag) {
                // Failure path only: give copies already in flight time to land.
                const unsigned long long t0 = globaltimer_ns();
                while (globaltimer_ns() - t0 < 1000000ull) {
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------- MMA issuer --
            constexpr uint32_t idesc = make_idesc_f16(128, BN, kMN ? 1 : 0);
            int it = 0, tl = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tl) {
                const int acc = tl & 1;
                if (!mbar_wait(&tempty_bar[acc], ((tl >> 1) & 1) ^ 1, abort_flag, args.status, kErrWaitAccum)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * Cfg::kAccStride;
                bool ok = true;
                for (int kb = 0; kb < num_kb; ++kb, ++it) {
                    const int st = it % S;
                    if (!mbar_wait(&full_bar[st], (it / S) & 1, abort_flag, args.status, kErrWaitFull) ||
                        (kQ4 && (!kRes || it < num_kb) &&
                         !mbar_wait(&ready_bar[st], (it / S) & 1, abort_flag, args.status, kErrWaitFull))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(kRes ? resA + kb * Cfg::kABytes : stages + st * Cfg::kStageBytes);
                    const uint32_t b_addr = smem_u32(stages + st * Cfg::kStageBytes + Cfg::kBOff);
#pragma unroll
                    for (int kk = 0; kk < Cfg::kBK / 16; ++kk) {
                        // K-major SW128: +32 B per 16 k inside the 128-B row.
                        // MN-major SW128: +2 KB per 16 k (two 8-row k groups of
                        // 1 KB); the two 64-element m halves are 8 KB apart (LBO).
                        const uint64_t adesc = kMN ? make_sdesc(a_addr + kk * 2048, 8192, 1024)
                                                   : make_sdesc(a_addr + kk * 32, 16, 1024);
                        const uint64_t bdesc = make_sdesc(b_addr + kk * 32, 16, 1024);
                        umma_f16(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0);
                    }
                    umma_commit(&empty_bar[st]);
                }
                // Published even after a failure: the barrier completes once all
                // issued MMAs are done, so TMEM is idle before it is freed.
                umma_commit(&tfull_bar[acc]);
                if (!ok) break;
            }
        }
    } else if (kQ4 && warp >= 12) {
        dequant(threadIdx.x - 384, dq_threads);
    } else if (warp >= 4 && warp < 12) {
        // ------------------------------------------------------ epilogue --
        const int eg = (warp - 4) >> 2;          // epilogue warpgroup == accumulator it drains
        const int bar_id = 1 + eg;
        const int q = warp & 3;                  // TMEM lane quadrant
        const int row = q * 32 + lane;           // D row of this thread
        const int et = (threadIdx.x - 128) & 127;  // 0..127 within the group
        float* sG = sE + eg * (Cfg::kGroupEpiBytes / 4);
        uint64_t* rbar = res_bar + 4 * eg;
        int tl = eg;                             // local tile index (this group takes tl = eg, eg+2, ...)
        int g_chunk = 0;                         // PW chunks processed by this group (buffer parity)
        // PW: chunks of 16 tokens, numbered g across this group's tiles
        // (BN/16 per tile).  A ring of R = 2A residual buffers: the load of
        // chunk g + A (possibly of the group's next tile) is issued while
        // chunk g is processed, once the store of chunk g - A has read its
        // buffer; the first A go out before the group's first accumulator is
        // complete.
        constexpr int CPT = kPW ? BN / Cfg::kChunk : 1;
        auto issue_res = [&](int gl) {  // residual chunk gl of this group's sequence, if any
            const int tt = blockIdx.x + (eg + 2 * (gl / CPT)) * gridDim.x;
            if (tt >= num_tiles) return;
            const int jb = gl % Cfg::kEpiRing;
            mbar_arrive_expect_tx(&rbar[jb], Cfg::kResBytes);
            tma_load_2d(sG + jb * (Cfg::kResBytes / 4), &tmap_res, &rbar[jb], (tt % args.m_tiles) * Cfg::kBM,
                        (tt / args.m_tiles) * BN + (gl % CPT) * Cfg::kChunk);
        };
        if (kPW && args.res != nullptr && et == 0) {
            for (int l = 0; l < Cfg::kEpiAhead; ++l) issue_res(l);
        }
        if (kQ4 && dq_help) dequant(kDqThreads + threadIdx.x - 128, dq_threads);
        for (int tile = blockIdx.x + eg * gridDim.x; tile < num_tiles; tile += 2 * gridDim.x, tl += 2) {
            const int acc = eg;
            // the tile's parameters are loaded first, then the accumulator awaited
            auto acc_ready = [&]() -> bool {
                bool r = mbar_wait(&tfull_bar[acc], (tl >> 1) & 1, abort_flag, args.status, kErrWaitAccum);
                r = !epi_bar_any(bar_id, !r || *abort_flag != 0);  // uniform over the group
                if (r) tc_fence_after();
                return r;
            };
            bool ok = true;
            const uint32_t t_row = tmem_base + acc * Cfg::kAccStride + (static_cast<uint32_t>(q * 32) << 16);
            const int mt = tile % args.m_tiles;
            const int nt = tile / args.m_tiles;
            if (kPW) {
                // The result is written in place (fp32) or to the chunk's fp16
                // buffer, and a TMA store sends it out.  Chunks past N load
                // zeros and store nothing (TMA clips).
                const int m0 = mt * Cfg::kBM;
                const int m = m0 + row;
                const int n_start = nt * BN;
                const bool mv = m < args.M;
                const float b = mv ? args.bias[m] : 0.f;
                const float al = (mv && args.snake_alpha) ? args.snake_alpha[m] : 0.f;
                const float iv = (mv && args.snake_alpha)
                                     ? (args.snake_inv ? args.snake_inv[m] : 1.0f / (al + 1e-9f))
                                     : 0.f;
                const bool has_res = args.res != nullptr;
                if (!(ok = acc_ready())) break;
#pragma unroll 1
                for (int ch = 0; ch < CPT; ++ch, ++g_chunk) {
                    const int j = g_chunk % Cfg::kEpiRing;
                    if (et == 0) {
                        // the store of chunk g - ahead has read its buffers
                        bulk_wait_read<Cfg::kEpiAhead - 1>();
                        if (has_res) issue_res(g_chunk + Cfg::kEpiAhead);
                    }
                    float v[16];
                    tmem_ld16(t_row + ch * Cfg::kChunk, v);
                    float* rbuf = sG + j * (Cfg::kResBytes / 4);
                    __half* obuf = reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(sG) +
                                                             Cfg::kEpiRing * Cfg::kResBytes + j * Cfg::kOut16Bytes);
                    bool w_ok = true;
                    if (has_res) w_ok = mbar_wait(&rbar[j], (g_chunk / Cfg::kEpiRing) & 1, abort_flag, args.status, kErrWaitFull);
                    if (w_ok) {
                        float r[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) r[i] = has_res ? rbuf[i * 128 + row] : 0.f;
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            float y = v[i] + b + r[i];
                            if (args.snake_alpha) y = snake(y, al, iv);
                            if (EPI == kEpiPW && args.out_f16) {
                                obuf[i * 128 + row] = __float2half_rn(y);
                            } else {
                                rbuf[i * 128 + row] = y;
                            }
                        }
                    }
                    fence_proxy_async_smem();
                    if (epi_bar_any(bar_id, !w_ok)) {  // uniform: some thread's residual never landed
                        ok = false;
                        break;
                    }
                    if (et == 0) {
                        tma_store_2d(&tmap_out, (EPI == kEpiPW && args.out_f16) ? static_cast<const void*>(obuf) : rbuf, m0,
                                     n_start + ch * Cfg::kChunk);
                        bulk_commit();
                    }
                }
            } else {
                // ConvT: 32-column chunks staged in smem, row stride 36 floats
                // (16-byte stores at the minimum 4 wavefronts), the previous
                // chunk's last column carried at index 3.  Then lane = output
                // token (column c), each warp takes (phase r, 4 couts) quads:
                //   y[(n*s + r)][co] = D[co*2s + r][c] + D[co*2s + s + r][c-1] + b[co]
                // (the second term absent at a sequence start), reads along
                // lanes without bank conflicts, one 16-byte store per quad.
                const int s = args.s;
                const int co_lo = mt * args.cpt;
                const int cpt = min(args.cpt, args.cout - co_lo);
                const int n_start = nt * (BN - 1) - 1;  // token of D column 0
                const int qpr = args.cpt / 4;           // cout quads per phase
                const int nquads = s * qpr;
                const int ew = et >> 5;                 // warp within the group
                float* out = static_cast<float*>(args.out);
                float4 bq[8];                           // bias of this warp's quads (nquads <= 32)
                int rco[8];                             // (phase << 16) | cout offset of each quad, -1 if none
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    // v8 (qpr == 2): quads k = 2i, 2i + 1 are couts 0-3 and 4-7 of phase ew + 4i
                    const int qd = args.v8 ? (ew + 4 * (k >> 1)) * 2 + (k & 1) : ew + 4 * k;
                    const int r = qd / qpr;
                    const int co = (qd - r * qpr) * 4;
                    const bool on = qd < nquads && co < cpt;
                    rco[k] = on ? (r << 16) | co : -1;
                    bq[k] = on ? *reinterpret_cast<const float4*>(args.bias + co_lo + co) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
                if (!(ok = acc_ready())) break;
                float carry = 0.f;
                float* rowp = sG + row * Cfg::kEpiLD;
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    float v[32];
                    tmem_ld16(t_row + c0, v);
                    tmem_ld16(t_row + c0 + 16, v + 16);
                    rowp[3] = carry;  // column c0 - 1
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        *reinterpret_cast<float4*>(rowp + 4 + 4 * j) = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                    carry = v[31];
                    epi_bar(bar_id);
                    const int c = c0 + lane;
                    const int n = n_start + c;
                    const int nl = n % args.seq_len;  // frame within its sequence
                    if (c >= 1 && c < BN && n < args.N && nl >= args.skip) {
                        const bool seq_start = nl == 0;
                        const size_t orow_n = static_cast<size_t>(n / args.seq_len) * (args.seq_len - args.skip) + (nl - args.skip);
                        float* orow = out + orow_n * s * args.cout + co_lo;  // y row (n*s + 0)
                        const float* sgl = sG + 4 + lane;
                        const int rs = 2 * s * Cfg::kEpiLD;                                  // next cout
                        if (args.v8) {
#pragma unroll
                            for (int k = 0; k < 8; k += 2) {
                                if (rco[k] < 0) continue;  // (quads k, k + 1 exist together)
                                const int r = rco[k] >> 16;
                                float4 y2[2];
#pragma unroll
                                for (int h = 0; h < 2; ++h) {
                                    const float* pa = sgl + ((4 * h) * 2 * s + r) * Cfg::kEpiLD;  // D[co*2s + r][c]
                                    const float* pb = pa + s * Cfg::kEpiLD - 1;  // D[co*2s + s + r][c - 1]
                                    float4 y;
                                    y.x = pa[0] + bq[k + h].x;
                                    y.y = pa[rs] + bq[k + h].y;
                                    y.z = pa[2 * rs] + bq[k + h].z;
                                    y.w = pa[3 * rs] + bq[k + h].w;
                                    if (!seq_start) {
                                        y.x += pb[0];
                                        y.y += pb[rs];
                                        y.z += pb[2 * rs];
                                        y.w += pb[3 * rs];
                                    }
                                    y2[h] = y;
                                }
                                st_global_v8(orow + r * args.cout, y2[0], y2[1]);
                            }
                        } else {
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            if (rco[k] < 0) continue;
                            const int r = rco[k] >> 16;
                            const int co = rco[k] & 0xffff;
                            const float* pa = sgl + (co * 2 * s + r) * Cfg::kEpiLD;  // D[co*2s + r][c]
                            const float* pb = pa + s * Cfg::kEpiLD - 1;               // D[co*2s + s + r][c - 1]
                            float4 y;
                            y.x = pa[0] + bq[k].x;
                            y.y = pa[rs] + bq[k].y;
                            y.z = pa[2 * rs] + bq[k].z;
                            y.w = pa[3 * rs] + bq[k].w;
                            if (!seq_start) {
                                y.x += pb[0];
                                y.y += pb[rs];
                                y.z += pb[2 * rs];
                                y.w += pb[3 * rs];
                            }
                            *reinterpret_cast<float4*>(orow + r * args.cout + co) = y;
                        }
                        }
                    }
                    epi_bar(bar_id);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty_bar[acc]);
            if (!ok) break;
        }
        if (kPW && et == 0) bulk_wait_all();  // stores done before the CTA's smem goes away
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace vxb
