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

// Residual-unit prologue.  Block = 32 channels x 8 thread rows; it covers
// kTT consecutive time steps of one sequence.  The needed input rows
// [t0 - 6d, t0 + kTT) are loaded once, Snake-activated (snake1) into shared
// memory, then every output applies the dilated causal taps, bias and
// snake2, and is stored as fp16.
constexpr int kPreTT = 32;

__global__ void __launch_bounds__(256) res_pre_kernel(const float* __restrict__ x, const float* __restrict__ a1,
                                                      const float* __restrict__ i1,
                                                      const float* __restrict__ w /*[C][7]*/,
                                                      const float* __restrict__ bias,
                                                      const float* __restrict__ a2,
                                                      const float* __restrict__ i2, __half* __restrict__ out,
                                                      int C, int T, int d) {
    extern __shared__ float sh[];  // [(kPreTT + 6d)][32]
    const int cx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + cx;
    const int t0 = blockIdx.y * kPreTT;
    const int b = blockIdx.z;
    const int halo = 6 * d;
    const int rows = kPreTT + halo;
    const bool cv = c < C;
    const float al1 = cv ? a1[c] : 0.f, iv1 = cv ? i1[c] : 0.f;
    const float* xb = x + static_cast<long long>(b) * T * C;
    for (int r = ty; r < rows; r += 8) {
        const int t = t0 - halo + r;
        float v = 0.f;  // causal zero padding (of snake1's output; snake(0) == 0)
        if (cv && t >= 0 && t < T) v = snake(xb[static_cast<long long>(t) * C + c], al1, iv1);
        sh[r * 32 + cx] = v;
    }
    __syncthreads();
    if (!cv) return;
    float wk[7];
#pragma unroll
    for (int k = 0; k < 7; ++k) wk[k] = w[c * 7 + k];
    const float bb = bias[c], al2 = a2[c], iv2 = i2[c];
    __half* ob = out + static_cast<long long>(b) * T * C;
    for (int tt = ty; tt < kPreTT; tt += 8) {
        const int t = t0 + tt;
        if (t >= T) break;
        float acc = bb;
#pragma unroll
        for (int k = 0; k < 7; ++k) acc = fmaf(sh[(tt + k * d) * 32 + cx], wk[k], acc);
        ob[static_cast<long long>(t) * C + c] = __float2half_rn(snake(acc, al2, iv2));
    }
}

// Final conv: y[b][t] = tanh(bias + sum_{c,k} w[c][k] * s[b*T + t + k - 6][c]).
// One warp per output sample; lanes stride over channels.
__global__ void __launch_bounds__(256) final_kernel(const float* __restrict__ s, const float* __restrict__ w /*[C][7]*/,
                                                    float bias, float* __restrict__ y, int C, int T,
                                                    long long total) {
    const int lane = threadIdx.x & 31;
    const long long warp_id = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) >> 5;
    const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
    for (long long n = warp_id; n < total; n += nwarps) {
        const int t = static_cast<int>(n % T);
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < 7; ++k) {
            const int st = t + k - 6;
            if (st < 0) continue;
            const float* row = s + (n + k - 6) * C;
            for (int c = lane; c < C; c += 32) acc = fmaf(row[c], w[c * 7 + k], acc);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) y[n] = tanhf(acc + bias);
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
