// Encoder-only kernels (the rest of the encoder runs on the decoder's
// residual-unit and GEMM kernels):
//   enc_head_kernel      head conv k7 (pad 3) 1 -> E channels on the waveform
//                        (encode_tensor, reference src/audio-vae.cpp:640-643).
//   snake_im2col_kernel  [Snake ->] im2col of a strided causal conv, fp16,
//                        the B operand of the conv as one pointwise GEMM
//                        (causal_conv1d + conv1d_mul_mat_impl, :476-493,
//                        :218-234).
//   latent_transpose_kernel  [B*T][L] -> [B][L][T] (ggml ne=[T, L]).
#pragma once

#include "common.cuh"

namespace vxb {

// x[b*L + t][c] = bias[c] + sum_k w[c][k] * a[b][t + k - 6], the waveform
// sample rounded to fp16 first as the reference's F16 mul_mat rounds its
// im2col rows (the weights are F16 values already).  One float4 of channels
// per thread; C % 4 == 0.
__global__ void enc_head_kernel(const float* __restrict__ audio, const float* __restrict__ w /*[C][7]*/,
                                const float* __restrict__ bias, float* __restrict__ x, int B, long long L,
                                int C) {
    grid_dep_sync();
    const int cq = C / 4;
    const long long total = static_cast<long long>(B) * L * cq;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % cq) * 4;
        const long long n = i / cq;
        const long long t = n % L;
        const float* a = audio + (n - t);  // this waveform
        float4 acc = *reinterpret_cast<const float4*>(bias + c);
#pragma unroll
        for (int k = 0; k < 7; ++k) {
            const long long src = t + k - 6;
            if (src < 0) continue;
            const float v = __half2float(__float2half_rn(a[src]));
            acc.x = fmaf(w[(c + 0) * 7 + k], v, acc.x);
            acc.y = fmaf(w[(c + 1) * 7 + k], v, acc.y);
            acc.z = fmaf(w[(c + 2) * 7 + k], v, acc.z);
            acc.w = fmaf(w[(c + 3) * 7 + k], v, acc.w);
        }
        *reinterpret_cast<float4*>(x + n * C + c) = acc;
    }
}

// col[(b*Lout + t)][ci*K + k] = f(x[b*Lin + t*s + k - lpad][ci]), zero where
// that row is before the sequence start (the causal left padding) or past
// its end; f = Snake(alpha, inv) or the identity (alpha == nullptr).  The
// column order ci*K + k (k fastest) is the memory order of the conv weight
// ([K, Cin, Cout] F16 or folded [K*Cin, Cout] Q4_0), so the conv is the GEMM
// y[n][co] = sum_j W[co][j] col[n][j] with the weight as stored.  One thread
// per (row, ci): its K values are one contiguous run of the row.
template <int K>
__global__ void snake_im2col_kernel(const float* __restrict__ x, const float* __restrict__ alpha,
                                    const float* __restrict__ inv, __half* __restrict__ col, int B, int Lin,
                                    int C, int s, int lpad, int Lout) {
    grid_dep_sync();
    const long long total = static_cast<long long>(B) * Lout * C;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int ci = static_cast<int>(i % C);
        const long long n = i / C;
        const int b = static_cast<int>(n / Lout);
        const int t = static_cast<int>(n - static_cast<long long>(b) * Lout);
        const float* xb = x + static_cast<long long>(b) * Lin * C + ci;
        const float al = alpha ? alpha[ci] : 0.f, iv = alpha ? inv[ci] : 0.f;
        __half v[K];
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const int src = t * s + k - lpad;
            float u = 0.f;
            if (src >= 0 && src < Lin) {
                u = xb[static_cast<long long>(src) * C];
                if (alpha) u = snake(u, al, iv);
            }
            v[k] = __float2half_rn(u);
        }
        __half* o = col + i * K;
        if constexpr (K % 8 == 0) {
#pragma unroll
            for (int j = 0; j < K / 8; ++j) reinterpret_cast<uint4*>(o)[j] = reinterpret_cast<const uint4*>(v)[j];
        } else if constexpr (K % 2 == 0) {
#pragma unroll
            for (int j = 0; j < K / 2; ++j) reinterpret_cast<__half2*>(o)[j] = __halves2half2(v[2 * j], v[2 * j + 1]);
        } else {
#pragma unroll
            for (int k = 0; k < K; ++k) o[k] = v[k];
        }
    }
}

// z[b][c][t] = y[b*T + t][c].
__global__ void latent_transpose_kernel(const float* __restrict__ y, float* __restrict__ z, int B, int T, int Lt) {
    grid_dep_sync();
    const long long total = static_cast<long long>(B) * Lt * T;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int t = static_cast<int>(i % T);
        const long long bc = i / T;
        const int c = static_cast<int>(bc % Lt);
        const long long b = bc / Lt;
        z[i] = y[(b * T + t) * Lt + c];
    }
}

}  // namespace vxb
