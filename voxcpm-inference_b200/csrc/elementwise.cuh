// Bandwidth-bound kernels around the tensor-core convs.
//
//   head_kernel      model.0: causal depthwise k7 conv of the latent
//                    (z [B][L][T], t fastest) -> fp16 [B*T][L], the B operand
//                    of the model.1 pointwise GEMM.
//   res_pre_kernel   residual-unit prologue: snake1 -> causal depthwise k7
//                    conv, dilation d (+bias) -> snake2 -> fp16 [N][C], the B
//                    operand of the unit's pointwise GEMM.
//   final_kernel     causal k7 conv C -> 1 over the (already Snake-activated)
//                    last stage, + bias, tanh -> waveform.
//   snake_kernel / q4_0_dequant_kernel: single-op kernels used by the C-ABI
//                    unit entry points.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace vxb {

// y[b*T + t][c] = b0[c] + sum_k w[c][k] * z[b][c][t + k - 6]   (reference
// depthwise_conv_l2_custom / depthwise_conv_custom with stride 1, dilation 1,
// padding 3: src = t + k*d - 2*pad).
// t_off: the first t_off frames of each z sequence are a streaming window's
// history: outputs start at frame t_off (out holds T - t_off frames per sequence).
__global__ void head_kernel(const float* __restrict__ z, const float* __restrict__ w /*[L][7]*/,
                            const float* __restrict__ bias, __half* __restrict__ out, int B, int L, int T,
                            int t_off) {
    grid_dep_sync();
    const int To = T - t_off;
    const long long total = static_cast<long long>(B) * To * L;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % L);
        const long long n = i / L;
        const int t = static_cast<int>(n % To) + t_off;
        const int b = static_cast<int>(n / To);
        const float* zc = z + (static_cast<long long>(b) * L + c) * T;
        float acc = bias[c];
#pragma unroll
        for (int k = 0; k < 7; ++k) {
            const int st = t + k - 6;
            if (st >= 0) acc = fmaf(zc[st], w[c * 7 + k], acc);
        }
        out[i] = __float2half_rn(acc);
    }
}

// Residual-unit prologue: snake1 -> causal depthwise k7 conv, dilation d
// (+ bias) -> snake2 -> fp16 [N][C], the B operand of the unit's pointwise
// GEMM.  Every thread owns one channel pair and a run of `run` outputs (a
// multiple of 7) of one sequence along one phase of the dilation
// (t = phase + j*d), and walks it with the 7 inputs its current output needs
// in a register window: each input row is read (8 bytes, a warp's pairs
// contiguous) and Snake-activated once, plus 6 warm-up rows per run -- the
// same overhead at every dilation -- and the next 7 rows are loaded while
// the current 7 are computed.  Rows before the sequence start are zero
// (causal padding; snake(0) == 0).  No shared memory.  The arithmetic per
// output is that of the reference unit (audio-vae.cpp:1481-1518): taps in
// order from the bias, one fma per tap and lane.  Requires C % 2 == 0.
// Three blocks per SM (80 registers): each thread's run is a chain bound by
// latency, so the SM's throughput grows with the threads it holds (at 96
// registers, two blocks, the 192/96-channel stages took 162 us instead of
// 152 at batch 256).
__host__ __device__ inline long long res_pre_threads(int C, int T, int B, int d, int run) {
    const long long J = (T + d - 1) / d;  // outputs per phase (at most)
    return static_cast<long long>(C / 2) * B * d * ((J + run - 1) / run);
}

// Run length: the longest of 56, 28, 14, 7 outputs that still gives every
// SM two blocks' worth of threads (short sequences get short runs).
inline int res_pre_run(int C, int T, int B, int d, int sms) {
    for (int run = 56; run > 7; run /= 2)
        if (res_pre_threads(C, T, B, d, run) >= 2LL * 256 * sms) return run;
    return 7;
}

// KW = false (the usual case): the thread index and every row offset inside
// one sequence fit 32 bits (the host checks), so the index arithmetic and the
// per-load / per-store address arithmetic are 32-bit; KW = true: 64-bit.
template <bool KW>
__global__ void __launch_bounds__(256, 3) res_pre_kernel(const float* __restrict__ x, const float* __restrict__ a1,
                                                      const float* __restrict__ i1,
                                                      const float* __restrict__ w /*[C][7]*/,
                                                      const float* __restrict__ bias,
                                                      const float* __restrict__ a2,
                                                      const float* __restrict__ i2, __half* __restrict__ out,
                                                      int C, int T, int B, int d, int run, int t_off) {
    using idx_t = typename std::conditional<KW, long long, int>::type;
    // T outputs per sequence; x holds T + t_off rows per sequence, the first
    // t_off of them a streaming window's history (output t reads row t + t_off)
    const int Tx = T + t_off;
    const int Q = C >> 1;
    const int J = (T + d - 1) / d;
    const int R = (J + run - 1) / run;
    const idx_t total = static_cast<idx_t>(Q) * B * d * R;
    const idx_t i = static_cast<idx_t>(blockIdx.x) * 256 + static_cast<idx_t>(threadIdx.x);
    const bool active = i < total;
    const int q = active ? static_cast<int>(i % Q) : 0;
    idx_t r = i / Q;
    const int jr = static_cast<int>(r % R);
    r /= R;
    const int phase = static_cast<int>(r % d);
    const int b = static_cast<int>(r / d);
    const int c = 2 * q;
    // per-channel constants are not written by earlier kernels: loaded
    // before the grid dependency wait, while the previous kernel finishes
    float2 wk[7];
#pragma unroll
    for (int k = 0; k < 7; ++k) wk[k] = make_float2(w[c * 7 + k], w[(c + 1) * 7 + k]);
    const float2 al1 = *reinterpret_cast<const float2*>(a1 + c);
    const float2 iv1 = *reinterpret_cast<const float2*>(i1 + c);
    const float2 bb = *reinterpret_cast<const float2*>(bias + c);
    const float2 al2 = *reinterpret_cast<const float2*>(a2 + c);
    const float2 iv2 = *reinterpret_cast<const float2*>(i2 + c);
    grid_dep_sync();
    if (!active) return;
    const float* xb = x + static_cast<long long>(b) * Tx * C + static_cast<long long>(t_off) * C + c;
    __half* ob = out + static_cast<long long>(b) * T * C + c;
    const int t_first = phase + (jr * run - 6) * d;  // row m of the run is t_first + m*d
    // rows -t_off .. T - 1 exist (one unsigned compare); rows before are the causal zero padding
    auto load = [&](int t) {
        return static_cast<unsigned>(t + t_off) < static_cast<unsigned>(Tx)
                   ? __ldg(reinterpret_cast<const float2*>(xb + static_cast<idx_t>(t) * C))
                   : make_float2(0.f, 0.f);
    };
    // window slot of row m is m % 7; rows 0..5 are the warm-up (before the first output)
    float2 win[7];
#pragma unroll
    for (int m = 0; m < 6; ++m) win[m] = load(t_first + m * d);
    float2 nxt[7];
#pragma unroll
    for (int s = 0; s < 7; ++s) nxt[s] = load(t_first + (6 + s) * d);
#pragma unroll
    for (int m = 0; m < 6; ++m) win[m] = snake2(win[m], al1, iv1);
#pragma unroll 1
    for (int g = 0; g < run; g += 7) {
        const int tg = t_first + (6 + g) * d;  // the group's first output row
        if (tg >= T) break;
        float2 cur[7];
#pragma unroll
        for (int s = 0; s < 7; ++s) cur[s] = nxt[s];
        if (g + 7 < run) {  // the next group's rows, loaded while this one computes
            const int tn = tg + 7 * d;  // its first row
            if (static_cast<unsigned>(tn + t_off) < static_cast<unsigned>(Tx) &&
                static_cast<unsigned>(tn + 6 * d + t_off) < static_cast<unsigned>(Tx)) {
                // all 7 rows inside the sequence (the usual case): no per-row checks
                const float* pn = xb + static_cast<idx_t>(tn) * C;
                const idx_t dC = static_cast<idx_t>(d) * C;
#pragma unroll
                for (int s = 0; s < 7; ++s) nxt[s] = __ldg(reinterpret_cast<const float2*>(pn + s * dC));
            } else {
#pragma unroll
                for (int s = 0; s < 7; ++s) nxt[s] = load(tn + s * d);
            }
        }
#pragma unroll
        for (int s = 0; s < 7; ++s) {
            // newest row m = 6 + g + s (slot (6 + s) % 7); tap k reads row m - 6 + k (slot (s + k) % 7)
            win[(6 + s) % 7] = snake2(cur[s], al1, iv1);
            float2 acc = bb;
#pragma unroll
            for (int k = 0; k < 7; ++k) acc = ffma2(win[(s + k) % 7], wk[k], acc);  // taps in order
            const int t = tg + s * d;
            if (t < T) {
                const float2 y = snake2(acc, al2, iv2);
                *reinterpret_cast<__half2*>(ob + static_cast<idx_t>(t) * C) = __floats2half2_rn(y.x, y.y);
            }
        }
    }
}

// Final conv: y[b][t] = tanh(bias + sum_{c,k} w[c][k] * s[b*T + t + k - 6][c])
// over the (already Snake-activated) last stage, held in fp16 (the reference
// rounds this conv's input to fp16 in its im2col + F16 mul_mat,
// audio-vae.cpp:218-234).  A block covers tt (64 or 128) time steps of one
// sequence: rows [t0 - 6, t0 + tt) are copied into shared memory as
// they are (fp16) by cp.async, rows before the sequence start zero-filled,
// with no register staging (the taps and the sums are all a thread holds).
// Each warp then computes 8 consecutive outputs at a time: lane = channel
// quad, the 14 rows they read are loaded once (8 bytes, widened to fp32),
// every lane accumulates its channels' share of all 8 sums, and one
// exchange of halves (xor 16, 8, 4) followed by xor 2, 1 leaves each sum
// complete on four lanes (9 shuffles for 8 outputs).  The kernel is
// issue-bound: the products are paired FMAs (fma.rn.f32x2), the even and
// odd channels of a quad summed in the two halves.  Requires C % 8 == 0 and
// C <= 128.
// Shared memory of final_kernel: tt + 6 rows of C fp16 channels.
__host__ __device__ inline size_t final_smem_bytes(int C, int tt) { return size_t(tt + 6) * C * 2; }

// t_off: s holds T + t_off rows per sequence, the first t_off a streaming
// window's history; y holds T outputs per sequence (output t reads rows up to t + t_off).
// CT > 0: the channel count as a compile-time constant (shared-memory
// offsets become immediates; 96 is the VoxCPM decoder's last stage); CT = 0
// takes it from the argument.
template <int CT>
__global__ void __launch_bounds__(256) final_kernel(const __half* __restrict__ s, const float* __restrict__ w /*[C][7]*/,
                                                    float bias, float* __restrict__ y, int c_arg, int T, int t_off,
                                                    int tt) {
    const int C = CT > 0 ? CT : c_arg;
    extern __shared__ uint4 fsh16[];  // [tt + 6][C] fp16, 8 channels per 16 bytes
    const int c8n = C / 8, c4n = C / 4;
    const int t0 = blockIdx.x * tt;
    const int b = blockIdx.y;
    const int rows = min(tt, T - t0) + 6;
    const __half* sb = s + static_cast<long long>(b) * (T + t_off) * C + static_cast<long long>(t_off) * C;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // each lane owns channel quad `lane` (C <= 128); the taps are constant:
    // read before the grid dependency wait
    float4 wk[7];
    const bool lv = lane < c4n;
#pragma unroll
    for (int k = 0; k < 7; ++k) {
        const int cc = lane * 4;
        wk[k] = lv ? make_float4(w[(cc + 0) * 7 + k], w[(cc + 1) * 7 + k], w[(cc + 2) * 7 + k], w[(cc + 3) * 7 + k])
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    grid_dep_sync();
    // thread -> 16-byte chunk cq = tid % 16 of rows tid / 16, + 16 per step (C <= 128: c8n <= 16)
    const int cq = threadIdx.x & 15;
    for (int r = threadIdx.x >> 4; r < tt + 6 && cq < c8n; r += 16) {
        const int i = r * c8n + cq;
        const int t = t0 - 6 + r;
        // rows before the sequence start (the causal zero padding) and past
        // the tile's last row are zero-filled
        const bool valid = t >= -t_off && r < rows;
        cp_async16(&fsh16[i], valid ? static_cast<const void*>(sb + static_cast<long long>(t) * C + cq * 8)
                                    : static_cast<const void*>(sb),
                   valid ? 16u : 0u);
    }
    cp_async_wait_all();
    __syncthreads();
    const uint2* fq = reinterpret_cast<const uint2*>(fsh16);  // [row][channel quad], 4 fp16 each
#pragma unroll 1
    for (int grp = 0; grp < tt / 64; ++grp) {
    const int q0 = warp * (tt / 8) + grp * 8;  // this group's outputs q0..q0+7 (smem rows q0..q0+13)
    if (t0 + q0 >= T) break;
    // paired FMAs: channels (0, 1) and (2, 3) of the quad accumulate in the
    // two lanes of a float2, added at the end
    float2 acc2[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc2[j] = make_float2(0.f, 0.f);
    // branch-free rows: every lane reads inside the tt + 6 staged rows (rows
    // past the tile are zero); lanes past the channel quads read quad 0 and
    // their sums are dropped before the reduction
    const int lq = lv ? lane : 0;
#pragma unroll
    for (int r = 0; r < 14; ++r) {
        const uint2 hq = fq[(q0 + r) * c4n + lq];
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&hq.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&hq.y));
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int k = r - j;  // tap of row q0 + r for output q0 + j
            if (k >= 0 && k < 7) {
                acc2[j] = ffma2(lo, make_float2(wk[k].x, wk[k].y), acc2[j]);
                acc2[j] = ffma2(hi, make_float2(wk[k].z, wk[k].w), acc2[j]);
            }
        }
    }
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = lv ? acc2[j].x + acc2[j].y : 0.f;
    // exchange halves: after xor 16 a lane keeps 4 sums (outputs 0-3 or 4-7),
    // after xor 8 two, after xor 4 one
    const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
    float a4[4], a2[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float give = h16 ? acc[i] : acc[i + 4];
        const float keep = h16 ? acc[i + 4] : acc[i];
        a4[i] = keep + __shfl_xor_sync(0xffffffffu, give, 16);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float give = h8 ? a4[i] : a4[i + 2];
        const float keep = h8 ? a4[i + 2] : a4[i];
        a2[i] = keep + __shfl_xor_sync(0xffffffffu, give, 8);
    }
    float sum;
    {
        const float give = h4 ? a2[0] : a2[1];
        const float keep = h4 ? a2[1] : a2[0];
        sum = keep + __shfl_xor_sync(0xffffffffu, give, 4);
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    const int j = (h16 ? 4 : 0) + (h8 ? 2 : 0) + (h4 ? 1 : 0);  // output this lane's sum belongs to
    const int t = t0 + q0 + j;
    if ((lane & 3) == 0 && t < T) y[static_cast<long long>(b) * T + t] = tanhf(sum + bias);
    }
}

// Failure probe: one thread waits on an mbarrier that nothing ever arrives
// on, through the same bounded wait every decode kernel uses, with a limit
// of limit_ns; the wait gives up, records kErrWaitFull in the status word
// and the kernel returns.  No fault, no trap: the context stays usable.
__global__ void wait_probe_kernel(int* status, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
    mbar_wait_for(&bar, 0, &abort_flag, status, kErrWaitFull, limit_ns);
}

// y[n][c] = snake(x[n][c]) for an fp32 [N][C] tensor.
__global__ void snake_kernel(const float* __restrict__ x, const float* __restrict__ alpha,
                             const float* __restrict__ inv, float* __restrict__ y, int C, long long total) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % C);
        const float iv = inv ? inv[c] : 1.0f / (alpha[c] + 1e-9f);
        y[i] = snake(x[i], alpha[c], iv);
    }
}

// Q4_0 blocks -> fp32, (nibble - 8) * d, one thread per block.
__global__ void q4_0_dequant_kernel(const uint8_t* __restrict__ blocks, float* __restrict__ out, long long nblk) {
    for (long long b = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; b < nblk;
         b += static_cast<long long>(gridDim.x) * blockDim.x) {
        const uint8_t* blk = blocks + b * 18;
        const float d = half_bits_to_float(static_cast<uint16_t>(blk[0] | (blk[1] << 8)));
        float* o = out + b * 32;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const uint32_t q = blk[2 + j];
            o[j] = static_cast<float>(static_cast<int>(q & 15u) - 8) * d;
            o[j + 16] = static_cast<float>(static_cast<int>(q >> 4) - 8) * d;
        }
    }
}

}  // namespace vxb
