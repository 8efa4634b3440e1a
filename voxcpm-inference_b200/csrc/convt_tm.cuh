// Transposed conv with the tokens as M (Q4_0 weights, long stages):
//
//   y[(n*s + r)][co] = b[co] + sum_ci x[n][ci] W[ci][co*2s + r] + sum_ci x[n-1][ci] W[ci][co*2s + s + r]
//
// (reference causal transpose conv, src/audio-vae.cpp:1642-1673 / :512-534:
// kernel 2s, stride s, the outputs of token n at rows n*s .. n*s + 2s - 1,
// cropped so that row n*s + r receives taps r of token n and s + r of token
// n - 1; the second term is absent at a sequence start).
//
// gemm_kernel<kAQ4MN, BN, kEpiConvT> puts the weights on M: the two taps of
// an output sample then sit in different TMEM lanes (different threads),
// and its epilogue gathers them through shared memory with two named
// barriers per 32-token chunk -- on the long stages (s = 5, 2) that gather,
// not the MMAs or HBM, sets the time.  Here the GEMM is transposed:
//   D[token][j] = sum_ci x[token][ci] * W[ci][j],   j = co*2s + r
// A = activations (fp16 [N][Cin], K-major, TMA), B = the weights of BN = 2s*cpt
// columns j (Q4_0 blocks TMA'd and dequantised once per CTA into a resident,
// K-major column of shared memory, as the resident-A GEMM does), D in TMEM
// with one token per lane: a thread holds every tap of its token, and tap
// s + r of token n - 1 is one __shfl_up from the lane below.  Each epilogue
// warp's 32 TMEM lanes are fed by their own 32-row TMA box that starts one
// token early (lane 0 is the previous warp's last token, the carry), so no
// value crosses warps: 124 new tokens per 128-row tile, no shared memory and
// no barrier in the epilogue.  Each warp stages its tokens' output rows in
// shared memory and sends them with one TMA store per tile: 16-byte stores
// scattered one per output row (stride s*Cout*4 between lanes) cost more
// than the rest of the kernel.
//
// Warp roles (512 threads): warp 0 lane 0 TMA producer; warp 1 TMEM owner,
// lane 0 issues the MMAs; warps 4-7 / 8-11 two epilogue warpgroups (group g
// drains accumulator g: every other tile); warps 12-15 dequantise the
// CTA's weight column (first tile only).  Every CTA keeps one j tile (the
// grid is a multiple of the j tiles) and walks token tiles.  Every wait is
// bounded; the CTA always frees its TMEM.
#pragma once

#include "gemm.cuh"

namespace vxb {

constexpr int kTmTokens = 124;   // new tokens per tile (4 warps x 31; each warp's lane 0 is a carry)
constexpr int kTmThreads = 512;

// Resident weight column: K <= 64 * tm_max_kb(s) (192 for stride 2, whose
// shared memory also holds the output staging, 384 otherwise).
__host__ __device__ constexpr int tm_max_kb(int s) { return s == 2 ? 3 : 6; }

struct ConvTmArgs {
    int K;                // Cin
    int N;                // tokens (batch * frames)
    int T;                // frames per sequence
    int s, cout, cpt;     // stride, Cout, couts per j tile (BN = 2s*cpt)
    int j_tiles, n_tiles; // tile grid: tile t -> j tile t % j_tiles, token tile t / j_tiles
    const float* bias;    // [Cout]
    float* out;           // fp32 [N*s][Cout]
    int* status;
};

// Shared memory: the resident weight column (KB k blocks of [BN j][64 k],
// K-major SW128: the dequantisers transpose the MN-major Q4_0 blocks once
// per CTA), then S stages of {A tile [128 tokens][64 k] K-major SW128 (16 KB),
// raw Q4_0 blocks (6 KB)}, then one output staging buffer per epilogue warp:
// its 31 tokens' 31*s output rows of 128 B (32 couts, 128-byte swizzle), sent
// by one TMA store per tile (kStaged: stride 2).  At stride 5 (16 couts, rows
// of 64 B) the staging would leave the mainloop two stages beside the 120 KB
// weight column (measured slower, with all 8 warps on every tile and rows of
// 32 B): its epilogue stores 32 bytes (8 couts, st.global.v8) per output row
// directly -- half the requests of 16-byte stores, b2 at batch 256 252 -> 183 us.
template <int SS, int CPT>
struct ConvTmCfg {
    static constexpr int BN = 2 * SS * CPT;
    static constexpr int kBTile = BN * 128;                // one k block of the weight column
    static constexpr int kResBytes = tm_max_kb(SS) * kBTile;
    static constexpr int kATile = 128 * 64 * 2;            // 16 KB
    static constexpr int kRawBytes = 6144;                 // >= kQ4MNRawBytes
    static constexpr int kStageBytes = kATile + kRawBytes;
    static constexpr bool kStaged = CPT * 4 == 128;
    static constexpr int kStgRows = 31 * SS;
    static constexpr int kStgWarpBytes = kStaged ? (kStgRows * 128 + 1023) / 1024 * 1024 : 0;
    static constexpr int kStgBytes = 8 * kStgWarpBytes;
    static constexpr int kFree = 220 * 1024 - kResBytes - kStgBytes - 1024 - kBarrierBytes;
    static constexpr int kStages = kFree / kStageBytes > 4 ? 4 : kFree / kStageBytes;
    static constexpr int kSmemBytes = kResBytes + kStages * kStageBytes + kStgBytes + 1024 + kBarrierBytes;
    static constexpr int kAccStride = BN <= 128 ? 128 : 256;
    static constexpr int kTmemCols = 2 * kAccStride;
    static_assert(BN % 32 == 0 && BN <= 160, "j tiles of whole Q4_0 blocks, at most 5 per k row");
    static_assert(kStages >= 2, "pipeline needs two stages");
    static_assert(kStgRows <= 256, "one TMA box per warp");
};

// tcgen05.ld of 32 lanes x 8 columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// tcgen05.ld of 32 lanes x 16 / 8 columns without the wait; tm_ld_wait()
// completes every load issued before it, and tm_pin() then ties each
// register to it (an empty volatile asm after the wait), so that no use of
// a loaded value is scheduled before the wait.
__device__ __forceinline__ void tm_ld16_nowait(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tm_ld8_nowait(uint32_t taddr, uint32_t* r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tm_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tm_pin(uint32_t& x) { asm volatile("" : "+r"(x)); }



// SS = stride s, CPT = couts per j tile (BN = 2 * SS * CPT weight columns).
template <int SS, int CPT>
__global__ void __launch_bounds__(kTmThreads, 1)
    convt_tm_kernel(const __grid_constant__ CUtensorMap tmap_x,   // fp16 [N][K], box {64 k, 32 tokens}, SW128
                    const __grid_constant__ CUtensorMap tmap_w,   // Q4_0 nibble rows, box {80 B, 64 k}
                    const __grid_constant__ CUtensorMap tmap_ws,  // Q4_0 scale rows, box {64 k, 5 blocks}
                    const __grid_constant__ CUtensorMap tmap_y,   // kStaged: fp32 [N*s][Cout], box {CPT, 31 s}, SW128
                    const ConvTmArgs args) {
    using Cfg = ConvTmCfg<SS, CPT>;
    constexpr int BN = Cfg::BN;
    constexpr int S = Cfg::kStages;
    extern __shared__ uint8_t tm_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tm_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* resB = smem;                       // the CTA's weight column, num_kb k blocks
    uint8_t* stages = smem + Cfg::kResBytes;
    uint8_t* stg = stages + S * Cfg::kStageBytes;  // kStaged: output staging, one buffer per epilogue warp
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(stg + Cfg::kStgBytes);  // A tile landed
    uint64_t* raw_bar = full_bar + S;     // Q4_0 raw blocks of a stage landed (first tile)
    uint64_t* ready_bar = raw_bar + S;    // k block of the weight column dequantised (first tile)
    uint64_t* empty_bar = ready_bar + S;  // stage consumed by the MMAs
    uint64_t* tfull_bar = empty_bar + S;  // accumulator [2] complete
    uint64_t* tempty_bar = tfull_bar + 2; // accumulator [2] drained (4 warps)
    uint64_t* done_bar = tempty_bar + 2;  // every MMA of the CTA complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_kb = (args.K + 63) / 64;
    const int num_tiles = args.j_tiles * args.n_tiles;
    const int jt = blockIdx.x % args.j_tiles;  // this CTA's j tile: the grid is a multiple of j_tiles
    const int j0 = jt * BN;                    // first weight column (a multiple of 32: whole Q4_0 blocks)
    const int M = 2 * SS * args.cout;          // weight columns of the layer

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&raw_bar[i], 1);
            mbar_init(&ready_bar[i], 4);  // the 4 dequantiser warps
            mbar_init(&empty_bar[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull_bar[i], 1);
            mbar_init(&tempty_bar[i], 4);  // the 4 warps of the group that drains the accumulator
        }
        mbar_init(done_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&tmap_x);
        prefetch_tmap(&tmap_w);
        prefetch_tmap(&tmap_ws);
        if (Cfg::kStaged) prefetch_tmap(&tmap_y);
    }
    if (warp == 1) tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ TMA producer --
            // The weight column's raw blocks travel with the first tile's k
            // steps; those of the first min(S, num_kb) go out before the grid
            // dependency wait (weights are not written by earlier kernels).
            auto issue_raw = [&](int st, int kb) {
                uint8_t* r_dst = stages + st * Cfg::kStageBytes + Cfg::kATile;
                mbar_arrive_expect_tx(&raw_bar[st], kQ4MNRawBytes);
                tma_load_2d(r_dst, &tmap_w, &raw_bar[st], (j0 >> 5) * 16, kb * 64);
                tma_load_2d(r_dst + kQ4MNScaleOff, &tmap_ws, &raw_bar[st], kb * 64, j0 >> 5);
            };
            const int n_pre = static_cast<int>(blockIdx.x) < num_tiles ? min(S, num_kb) : 0;
            for (int kb = 0; kb < n_pre; ++kb) issue_raw(kb, kb);
            grid_dep_sync();
            int it = 0;
            for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
                const int n0 = (tile / args.j_tiles) * kTmTokens;
                bool ok = true;
                for (int kb = 0; kb < num_kb; ++kb, ++it) {
                    const int st = it % S;
                    if (it >= n_pre) {
                        if (!mbar_wait(&empty_bar[st], ((it / S) & 1) ^ 1, abort_flag, args.status, kErrWaitEmpty)) {
                            ok = false;
                            break;
                        }
                        if (it < num_kb) issue_raw(st, kb);
                    }
                    // four 32-row boxes: warp q's TMEM lanes take tokens
                    // n0 + 31q - 1 .. n0 + 31q + 30 (row -1 reads as zero)
                    uint8_t* a_dst = stages + st * Cfg::kStageBytes;
                    mbar_arrive_expect_tx(&full_bar[st], Cfg::kATile);
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        tma_load_2d(a_dst + q * 4096, &tmap_x, &full_bar[st], kb * 64, n0 + 31 * q - 1);
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
    } else if (warp >= 12) {
        // ------------------------------------------------- dequantisers --
        // First tile only: k block kb of the weight column, K-major SW128
        // [BN j][64 k] (the B operand's layout).  Item i -> k row kl = i % 64
        // and Q4_0 block bi = i / 64 of the BN / 32 in the row; its 32 values
        // (consecutive j) are transposed into 32 two-byte stores, once per CTA.
        const int t = threadIdx.x - 384;
        const __half zero = __float2half_rn(0.f);
        for (int kb = 0; kb < num_kb && static_cast<int>(blockIdx.x) < num_tiles; ++kb) {
            const int st = kb % S;
            if (!mbar_wait(&raw_bar[st], (kb / S) & 1, abort_flag, args.status, kErrWaitFull)) break;
            const uint8_t* raw = stages + st * Cfg::kStageBytes + Cfg::kATile;
            const __half* sc = reinterpret_cast<const __half*>(raw + kQ4MNScaleOff);
            uint8_t* b_dst = resB + kb * Cfg::kBTile;
            for (int i = t; i < 64 * (BN / 32); i += 128) {
                const int kl = i & 63, bi = i >> 6;
                const bool valid = j0 + bi * 32 < M && kb * 64 + kl < args.K;
                const __half2 d2 = __half2half2(valid ? sc[bi * 64 + kl] : zero);
                const uint4 q = *reinterpret_cast<const uint4*>(raw + kl * kQ4MNNibBox + bi * 16);
                const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int c = 0; c < 4; ++c) {  // word c: columns bi*32 + 8c .. + 7
                    const uint4 h8 = q4_dequant8_split(qw[c], d2);
                    const __half* hv = reinterpret_cast<const __half*>(&h8);
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        *reinterpret_cast<__half*>(b_dst + sw128_kmajor_off(bi * 32 + c * 8 + e, kl)) = hv[e];
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ready_bar[st]);
        }
    }
    else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------- MMA issuer --
            // A (tokens x k) and B (weight columns x k) both K-major.
            constexpr uint32_t idesc = make_idesc_f16(128, BN, 0);
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
                        (it < num_kb &&
                         !mbar_wait(&ready_bar[st], (it / S) & 1, abort_flag, args.status, kErrWaitFull))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(stages + st * Cfg::kStageBytes);
                    const uint32_t b_addr = smem_u32(resB + kb * Cfg::kBTile);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        // K-major SW128: +32 B per 16 k inside the 128-B rows
                        const uint64_t adesc = make_sdesc(a_addr + kk * 32, 16, 1024);
                        const uint64_t bdesc = make_sdesc(b_addr + kk * 32, 16, 1024);
                        umma_f16(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0);
                    }
                    umma_commit(&empty_bar[st]);
                }
                // published even after a failure: it completes once the issued MMAs are done
                umma_commit(&tfull_bar[acc]);
                if (!ok) break;
            }
        }
    } else if (warp >= 4 && warp < 12) {
        // ------------------------------------------------------- epilogue --
        // Lane l of warp q (TMEM quadrant q = warp % 4) holds token
        // n = n0 + 31q + l - 1 (lane 0: the carry, whose taps s..2s-1 only
        // feed lane 1).  Per 4 couts, the 8s columns co*2s + r come from TMEM;
        // tap s + r of token n - 1 is one shuffle up; y = (tap r + b) + tap
        // s + r of n - 1 (absent at a sequence start).  The warp writes its
        // 31 tokens' rows into its staging buffer (row (l - 1)*s + r) and
        // sends them with one TMA store per tile (kStaged), or stores each
        // row's 16 bytes directly.  Group eg drains accumulator eg (the CTA's
        // tiles eg, eg + 2, ...).
        const int eg = (warp - 4) >> 2;
        const int q = warp & 3;
        const int co_lo = jt * CPT;                // the host requires Cout % CPT == 0
        uint8_t* stg_w = stg + (warp - 4) * Cfg::kStgWarpBytes;
        grid_dep_sync();                           // the output may be a buffer the previous kernel still reads
        int tl = eg;
        for (int tile = blockIdx.x + eg * gridDim.x; tile < num_tiles; tile += 2 * gridDim.x, tl += 2) {
            const int acc = eg;
            const bool ok = mbar_wait(&tfull_bar[acc], (tl >> 1) & 1, abort_flag, args.status, kErrWaitAccum);
            if (__any_sync(0xffffffffu, !ok)) break;
            tc_fence_after();
            const int n0 = (tile / args.j_tiles) * kTmTokens;
            const int n = n0 + 31 * q + lane - 1;
            const bool tok = lane >= 1 && n < args.N;
            const bool seq_start = tok && n % args.T == 0;
            float* orow = args.out + (static_cast<size_t>(tok ? n : 0) * SS) * args.cout + co_lo;  // row n*s
            const uint32_t t_row = tmem_base + acc * Cfg::kAccStride + (static_cast<uint32_t>(q * 32) << 16);
            if (Cfg::kStaged) {
                if (lane == 0) bulk_wait_read<0>();  // the warp's store of its previous tile has read the buffer
                __syncwarp();
            }
            // kStaged: one cout quad per TMEM wait, 16-byte chunks into the
            // staging rows; direct: two quads per wait and one 32-byte store
            // per output row (8 consecutive couts)
            constexpr int QG = Cfg::kStaged ? 1 : 2;
            static_assert((CPT / 4) % QG == 0, "quad groups");
#pragma unroll 1
            for (int cq0 = 0; cq0 < CPT / 4; cq0 += QG) {
                uint32_t vr[QG * 8 * SS];
#pragma unroll
                for (int c = 0; c + 16 <= QG * 8 * SS; c += 16) tm_ld16_nowait(t_row + cq0 * 8 * SS + c, vr + c);
                if ((QG * 8 * SS) % 16)
                    tm_ld8_nowait(t_row + cq0 * 8 * SS + (QG * 8 * SS) / 16 * 16, vr + (QG * 8 * SS) / 16 * 16);
                tm_ld_wait();
#pragma unroll
                for (int c = 0; c < QG * 8 * SS; ++c) tm_pin(vr[c]);
                float4 bq[QG];
#pragma unroll
                for (int g = 0; g < QG; ++g) bq[g] = __ldg(reinterpret_cast<const float4*>(args.bias + co_lo) + cq0 + g);
#pragma unroll
                for (int r = 0; r < SS; ++r) {
                    float4 y[QG];
#pragma unroll
                    for (int g = 0; g < QG; ++g) {
                        const uint32_t* v = vr + g * 8 * SS;  // columns of quad cq0 + g
                        const float p0 = __shfl_up_sync(0xffffffffu, __uint_as_float(v[0 * 2 * SS + SS + r]), 1);
                        const float p1 = __shfl_up_sync(0xffffffffu, __uint_as_float(v[1 * 2 * SS + SS + r]), 1);
                        const float p2 = __shfl_up_sync(0xffffffffu, __uint_as_float(v[2 * 2 * SS + SS + r]), 1);
                        const float p3 = __shfl_up_sync(0xffffffffu, __uint_as_float(v[3 * 2 * SS + SS + r]), 1);
                        y[g].x = __uint_as_float(v[0 * 2 * SS + r]) + bq[g].x;
                        y[g].y = __uint_as_float(v[1 * 2 * SS + r]) + bq[g].y;
                        y[g].z = __uint_as_float(v[2 * 2 * SS + r]) + bq[g].z;
                        y[g].w = __uint_as_float(v[3 * 2 * SS + r]) + bq[g].w;
                        if (!seq_start) {
                            y[g].x += p0;
                            y[g].y += p1;
                            y[g].z += p2;
                            y[g].w += p3;
                        }
                    }
                    if (Cfg::kStaged) {
                        // row (lane - 1)*s + r of the box, chunk cq0 (128-byte swizzle)
                        const uint32_t row = static_cast<uint32_t>((lane - 1) * SS + r);
                        if (lane >= 1)
                            *reinterpret_cast<float4*>(stg_w + row * 128u +
                                                       (((static_cast<uint32_t>(cq0) ^ row) & 7u) << 4)) = y[0];
                    } else if (tok) {
                        st_global_v8(orow + r * args.cout + cq0 * 4, y[0], y[QG - 1]);
                    }
                }
            }
            // accumulator read: the MMAs of tile tl + 2 may reuse it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty_bar[acc]);
            if (Cfg::kStaged) {
                fence_proxy_async_smem();
                __syncwarp();
                // rows past the last token fall outside the tensor and are not written
                if (lane == 0 && n0 + 31 * q < args.N) {
                    tma_store_2d(&tmap_y, stg_w, co_lo, (n0 + 31 * q) * SS);
                    bulk_commit();
                }
            }
        }
        if (Cfg::kStaged && lane == 0) bulk_wait_all();  // stores done before the CTA's shared memory goes away
    }

    if (warp == 1 && lane == 0) {
        // every MMA this CTA issued has completed before TMEM is freed (also
        // on the failure paths, where no epilogue waited for the last ones)
        umma_commit(done_bar);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(done_bar, 0) && globaltimer_ns() - t0 < kWaitNs) {
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace vxb
