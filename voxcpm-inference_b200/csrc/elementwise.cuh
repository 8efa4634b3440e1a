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

#include "common.cuh"

namespace vxb {

// y[b*T + t][c] = b0[c] + sum_k w[c][k] * z[b][c][t + k - 6]   (reference
// depthwise_conv_l2_custom / depthwise_conv_custom with stride 1, dilation 1,
// padding 3: src = t + k*d - 2*pad).
__global__ void head_kernel(const float* __restrict__ z, const float* __restrict__ w /*[L][7]*/,
                            const float* __restrict__ bias, __half* __restrict__ out, int B, int L, int T) {
    grid_dep_sync();
    const long long total = static_cast<long long>(B) * T * L;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % L);
        const long long n = i / L;
        const int t = static_cast<int>(n % T);
        const int b = static_cast<int>(n / T);
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

// Residual-unit prologue.  A block covers CT channels (CT/4 threads x
// float4) and `tt` (<= kPreTT) time steps of one sequence.  The input rows
// [t0 - 6d, t0 + tt) are copied into shared memory with 16-byte cp.async
// (zero-filled before the sequence start: causal padding, snake(0) == 0) and
// Snake-activated (snake1) in place by the thread that copied them; every
// output then applies the 7 dilated causal taps, bias and snake2 and is
// stored as fp16.  CT = 64 when C is a multiple of 64, else 32 (C = 96 keeps
// every thread busy).  Requires C % 4 == 0.
constexpr int kPreTT = 128;

__host__ __device__ constexpr size_t res_pre_smem(int d, int tt = kPreTT, int ct = 64) {
    return sizeof(float) * (tt + 6 * d) * ct;
}

template <int CT>
__global__ void __launch_bounds__(256) res_pre_kernel(const float* __restrict__ x, const float* __restrict__ a1,
                                                      const float* __restrict__ i1,
                                                      const float* __restrict__ w /*[C][7]*/,
                                                      const float* __restrict__ bias,
                                                      const float* __restrict__ a2,
                                                      const float* __restrict__ i2, __half* __restrict__ out,
                                                      int C, int T, int d, int tt) {
    constexpr int CG = CT / 4;    // threads across channels
    constexpr int RG = 256 / CG;  // threads across rows
    extern __shared__ float4 sh4[];  // [(tt + 6d)][CG]
    const int cx = threadIdx.x % CG, ry = threadIdx.x / CG;
    const int c = blockIdx.x * CT + cx * 4;
    const int t0 = blockIdx.y * tt;
    const int b = blockIdx.z;
    const int halo = 6 * d;
    const int rows = min(tt, T - t0) + halo;
    const bool cv = c < C;
    const float* xb = x + static_cast<long long>(b) * T * C;
    {
        // the per-channel parameters are not written by earlier kernels: pull
        // this block's lines into L2 while the previous kernel finishes
        const int c0 = blockIdx.x * CT, nc = min(CT, C - c0), i = threadIdx.x;
        if (i < 10) {
            const float* v = i < 2 ? a1 : i < 4 ? i1 : i < 6 ? bias : i < 8 ? a2 : i2;
            if ((i & 1) * 32 < nc) prefetch_l2(v + c0 + (i & 1) * 32);
        } else if (i < 10 + 2 * CT * 7 / 64) {
            if ((i - 10) * 32 < nc * 7) prefetch_l2(w + c0 * 7 + (i - 10) * 32);
        }
    }
    grid_dep_sync();
    for (int r = ry; r < rows; r += RG) {
        const int t = t0 - halo + r;
        const bool ok = cv && t >= 0;
        cp_async16(&sh4[r * CG + cx], ok ? xb + static_cast<long long>(t) * C + c : xb, ok ? 16u : 0u);
    }
    cp_async_wait_all();
    if (cv) {
        const float4 al1 = *reinterpret_cast<const float4*>(a1 + c);
        const float4 iv1 = *reinterpret_cast<const float4*>(i1 + c);
        for (int r = ry; r < rows; r += RG) sh4[r * CG + cx] = snake4(sh4[r * CG + cx], al1, iv1);
    }
    __syncthreads();
    if (!cv) return;
    float2 wlo[7], whi[7];
#pragma unroll
    for (int k = 0; k < 7; ++k) {
        wlo[k] = make_float2(w[(c + 0) * 7 + k], w[(c + 1) * 7 + k]);
        whi[k] = make_float2(w[(c + 2) * 7 + k], w[(c + 3) * 7 + k]);
    }
    const float4 bb = *reinterpret_cast<const float4*>(bias + c);
    const float4 al2 = *reinterpret_cast<const float4*>(a2 + c);
    const float4 iv2 = *reinterpret_cast<const float4*>(i2 + c);
    __half* ob = out + static_cast<long long>(b) * T * C;
    for (int q = ry; q < tt; q += RG) {
        const int t = t0 + q;
        if (t >= T) break;
        float2 lo = make_float2(bb.x, bb.y), hi = make_float2(bb.z, bb.w);
#pragma unroll
        for (int k = 0; k < 7; ++k) {  // taps in order, one fma per tap and lane
            const float4 u = sh4[(q + k * d) * CG + cx];
            lo = ffma2(make_float2(u.x, u.y), wlo[k], lo);
            hi = ffma2(make_float2(u.z, u.w), whi[k], hi);
        }
        const float4 y = snake4(make_float4(lo.x, lo.y, hi.x, hi.y), al2, iv2);
        const __half2 h01 = __floats2half2_rn(y.x, y.y);
        const __half2 h23 = __floats2half2_rn(y.z, y.w);
        uint2 pk;
        pk.x = *reinterpret_cast<const uint32_t*>(&h01);
        pk.y = *reinterpret_cast<const uint32_t*>(&h23);
        *reinterpret_cast<uint2*>(ob + static_cast<long long>(t) * C + c) = pk;
    }
}

// Channel tile of res_pre_kernel for C channels.
inline int res_pre_ct(int C) { return C % 64 == 0 ? 64 : 32; }

// Time tile of res_pre_kernel: the largest of 128/64/32 that still gives at
// least two blocks per SM.
inline int res_pre_tt(int C, int T, int B, int sms) {
    const long long ct = (C + res_pre_ct(C) - 1) / res_pre_ct(C);
    for (int tt = kPreTT; tt > 32; tt /= 2)
        if (ct * ((T + tt - 1) / tt) * B >= 2LL * sms) return tt;
    return 32;
}

// Final conv: y[b][t] = tanh(bias + sum_{c,k} w[c][k] * s[b*T + t + k - 6][c])
// over the (already Snake-activated) last stage.  A block covers kFinTT time
// steps of one sequence: rows [t0 - 6, t0 + kFinTT) are staged in shared
// memory with 16-byte loads.  Each warp then computes 8 consecutive outputs
// at once: lane = channel quad, the 14 rows they read are loaded once, every
// lane accumulates its channels' share of all 8 sums, and one exchange of
// halves (xor 16, 8, 4) followed by xor 2, 1 leaves each sum complete on four
// lanes (9 shuffles for 8 outputs).  Requires C % 4 == 0 and C <= 128.
constexpr int kFinTT = 64;

__global__ void __launch_bounds__(256) final_kernel(const float* __restrict__ s, const float* __restrict__ w /*[C][7]*/,
                                                    float bias, float* __restrict__ y, int C, int T) {
    extern __shared__ float4 fsh4[];  // [(kFinTT + 6)][C/4]
    const int c4n = C / 4;
    const int t0 = blockIdx.x * kFinTT;
    const int b = blockIdx.y;
    const int rows = min(kFinTT, T - t0) + 6;
    const float* sb = s + static_cast<long long>(b) * T * C;
    if (threadIdx.x * 32 < C * 7) prefetch_l2(w + threadIdx.x * 32);  // taps: constant, into L2 before the wait
    grid_dep_sync();
    constexpr int kMaxLd = ((kFinTT + 6) * 32 + 255) / 256;  // float4 per thread for C <= 128
    float4 v[kMaxLd];
#pragma unroll
    for (int j = 0; j < kMaxLd; ++j) {  // every load issued before any is stored
        const int i = threadIdx.x + j * 256;
        const int r = i / c4n, cq = i - r * c4n;
        const int t = t0 - 6 + r;
        v[j] = (i < rows * c4n && t >= 0)
                   ? __ldg(reinterpret_cast<const float4*>(sb + static_cast<long long>(t) * C) + cq)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < kMaxLd; ++j) {
        const int i = threadIdx.x + j * 256;
        if (i < rows * c4n) fsh4[i] = v[j];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // each lane owns channel quad `lane` (C <= 128)
    float4 wk[7];
    const bool lv = lane < c4n;
#pragma unroll
    for (int k = 0; k < 7; ++k) {
        const int cc = lane * 4;
        wk[k] = lv ? make_float4(w[(cc + 0) * 7 + k], w[(cc + 1) * 7 + k], w[(cc + 2) * 7 + k], w[(cc + 3) * 7 + k])
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int q0 = warp * 8;  // this warp's outputs q0..q0+7 (smem rows q0..q0+13)
    if (t0 + q0 >= T) return;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
    for (int r = 0; r < 14; ++r) {
        const float4 u = (lv && q0 + r < rows) ? fsh4[(q0 + r) * c4n + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int k = r - j;  // tap of row q0 + r for output q0 + j
            if (k >= 0 && k < 7) {
                acc[j] = fmaf(u.x, wk[k].x, acc[j]);
                acc[j] = fmaf(u.y, wk[k].y, acc[j]);
                acc[j] = fmaf(u.z, wk[k].z, acc[j]);
                acc[j] = fmaf(u.w, wk[k].w, acc[j]);
            }
        }
    }
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
