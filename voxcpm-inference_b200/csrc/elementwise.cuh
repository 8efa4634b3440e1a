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

// Residual-unit prologue.  A block covers 64 channels (16 threads x float4)
// and `tt` (<= kPreTT) time steps of one sequence.  The input rows
// [t0 - 6d, t0 + tt) are loaded once with 16-byte loads (all of a thread's
// loads issued before any is used) and Snake-activated (snake1) into shared
// memory; every output then applies the 7 dilated causal taps, bias and
// snake2 and is stored as fp16.  Requires C % 4 == 0.
constexpr int kPreTT = 128;
constexpr int kPreMaxRows = (kPreTT + 54 + 15) / 16;  // rows per thread for d <= 9

__host__ __device__ constexpr size_t res_pre_smem(int d, int tt = kPreTT) { return sizeof(float) * (tt + 6 * d) * 64; }

__global__ void __launch_bounds__(256) res_pre_kernel(const float* __restrict__ x, const float* __restrict__ a1,
                                                      const float* __restrict__ i1,
                                                      const float* __restrict__ w /*[C][7]*/,
                                                      const float* __restrict__ bias,
                                                      const float* __restrict__ a2,
                                                      const float* __restrict__ i2, __half* __restrict__ out,
                                                      int C, int T, int d, int tt) {
    extern __shared__ float4 sh4[];  // [(tt + 6d)][16]
    const int cx = threadIdx.x & 15, ry = threadIdx.x >> 4;  // 16 channel groups x 16 rows
    const int c = blockIdx.x * 64 + cx * 4;
    const int t0 = blockIdx.y * tt;
    const int b = blockIdx.z;
    const int halo = 6 * d;
    const int rows = min(tt, T - t0) + halo;
    const bool cv = c < C;
    const float* xb = x + static_cast<long long>(b) * T * C;
    float4 v[kPreMaxRows];
#pragma unroll
    for (int i = 0; i < kPreMaxRows; ++i) {
        const int r = ry + 16 * i;
        const int t = t0 - halo + r;
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);  // causal zero padding (snake(0) == 0)
        if (cv && r < rows && t >= 0) v[i] = __ldg(reinterpret_cast<const float4*>(xb + static_cast<long long>(t) * C + c));
    }
    if (cv) {
        const float4 al1 = *reinterpret_cast<const float4*>(a1 + c);
        const float4 iv1 = *reinterpret_cast<const float4*>(i1 + c);
#pragma unroll
        for (int i = 0; i < kPreMaxRows; ++i) {
            const int r = ry + 16 * i;
            if (r >= rows) break;
            float4 u = v[i];
            u.x = snake(u.x, al1.x, iv1.x);
            u.y = snake(u.y, al1.y, iv1.y);
            u.z = snake(u.z, al1.z, iv1.z);
            u.w = snake(u.w, al1.w, iv1.w);
            sh4[r * 16 + cx] = u;
        }
    }
    __syncthreads();
    if (!cv) return;
    float4 wk[7];
#pragma unroll
    for (int k = 0; k < 7; ++k)
        wk[k] = make_float4(w[(c + 0) * 7 + k], w[(c + 1) * 7 + k], w[(c + 2) * 7 + k], w[(c + 3) * 7 + k]);
    const float4 bb = *reinterpret_cast<const float4*>(bias + c);
    const float4 al2 = *reinterpret_cast<const float4*>(a2 + c);
    const float4 iv2 = *reinterpret_cast<const float4*>(i2 + c);
    __half* ob = out + static_cast<long long>(b) * T * C;
    for (int q = ry; q < tt; q += 16) {
        const int t = t0 + q;
        if (t >= T) break;
        float4 acc = bb;
#pragma unroll
        for (int k = 0; k < 7; ++k) {
            const float4 u = sh4[(q + k * d) * 16 + cx];
            acc.x = fmaf(u.x, wk[k].x, acc.x);
            acc.y = fmaf(u.y, wk[k].y, acc.y);
            acc.z = fmaf(u.z, wk[k].z, acc.z);
            acc.w = fmaf(u.w, wk[k].w, acc.w);
        }
        const __half2 h01 = __floats2half2_rn(snake(acc.x, al2.x, iv2.x), snake(acc.y, al2.y, iv2.y));
        const __half2 h23 = __floats2half2_rn(snake(acc.z, al2.z, iv2.z), snake(acc.w, al2.w, iv2.w));
        uint2 pk;
        pk.x = *reinterpret_cast<const uint32_t*>(&h01);
        pk.y = *reinterpret_cast<const uint32_t*>(&h23);
        *reinterpret_cast<uint2*>(ob + static_cast<long long>(t) * C + c) = pk;
    }
}

// Time tile of res_pre_kernel: the largest of 128/64/32 that still gives at
// least two blocks per SM.
inline int res_pre_tt(int C, int T, int B, int sms) {
    const long long ct = (C + 63) / 64;
    for (int tt = kPreTT; tt > 32; tt /= 2)
        if (ct * ((T + tt - 1) / tt) * B >= 2LL * sms) return tt;
    return 32;
}

// Final conv: y[b][t] = tanh(bias + sum_{c,k} w[c][k] * s[b*T + t + k - 6][c])
// over the (already Snake-activated) last stage.  A block covers kFinTT time
// steps of one sequence: rows [t0 - 6, t0 + kFinTT) are staged in shared
// memory with 16-byte loads; each warp then reduces one output at a time over
// channels (lanes) and taps.  Requires C % 4 == 0 and C <= 128.
constexpr int kFinTT = 64;

__global__ void __launch_bounds__(256) final_kernel(const float* __restrict__ s, const float* __restrict__ w /*[C][7]*/,
                                                    float bias, float* __restrict__ y, int C, int T) {
    extern __shared__ float4 fsh4[];  // [(kFinTT + 6)][C/4]
    const int c4n = C / 4;
    const int t0 = blockIdx.x * kFinTT;
    const int b = blockIdx.y;
    const int rows = min(kFinTT, T - t0) + 6;
    const float* sb = s + static_cast<long long>(b) * T * C;
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
    // each lane owns channel quads lane, lane + 32, ... (C <= 128: at most one)
    float4 wk[7];
    const bool lv = lane < c4n;
#pragma unroll
    for (int k = 0; k < 7; ++k) {
        const int cc = lane * 4;
        wk[k] = lv ? make_float4(w[(cc + 0) * 7 + k], w[(cc + 1) * 7 + k], w[(cc + 2) * 7 + k], w[(cc + 3) * 7 + k])
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int tt = warp; tt < kFinTT; tt += 8) {
        const int t = t0 + tt;
        if (t >= T) break;
        float acc = 0.f;
        if (lv) {
#pragma unroll
            for (int k = 0; k < 7; ++k) {
                const float4 v = fsh4[(tt + k) * c4n + lane];
                acc = fmaf(v.x, wk[k].x, acc);
                acc = fmaf(v.y, wk[k].y, acc);
                acc = fmaf(v.z, wk[k].z, acc);
                acc = fmaf(v.w, wk[k].w, acc);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) y[static_cast<long long>(b) * T + t] = tanhf(acc + bias);
    }
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
