// Encoder-only kernels (the rest of the encoder runs on the decoder's
// residual-unit and GEMM kernels):
//   enc_head_kernel      head conv k7 (pad 3) 1 -> E channels on the waveform
//                        (encode_tensor, reference src/audio-vae.cpp:640-643).
//   im2col_rows_kernel   im2col of a strided causal conv over its fp16 input
//                        (the previous kernel's epilogue applied the Snake),
//                        the B operand of the conv as one pointwise GEMM
//                        (causal_conv1d + conv1d_mul_mat_impl, :476-493,
//                        :218-234); permute_ck_kernel reorders the conv
//                        weight to match once.
//   latent_transpose_kernel  [B*T][L] -> [B][L][T] (ggml ne=[T, L]).
#pragma once

#include "common.cuh"

namespace vxb {

// x[b*L + t][c] = bias[c] + sum_k w[c][k] * a[b][t + k - 6], the waveform
// sample rounded to fp16 first as the reference's F16 mul_mat rounds its
// im2col rows (the weights are F16 values already).  A block is C/4 channel
// quads x G token groups (G = blockDim / (C/4)); a thread keeps its quad's 28
// taps in registers and walks a run of kHeadRun consecutive tokens with the
// 7 samples they need in a sliding register window (one new sample per
// token, the same address for the whole group).  The group's C/4 float4
// stores cover one contiguous token row.  C % 4 == 0, C / 4 <= blockDim.
constexpr int kHeadRun = 32;

__global__ void enc_head_kernel(const float* __restrict__ audio, const float* __restrict__ w /*[C][7]*/,
                                const float* __restrict__ bias, float* __restrict__ x, int B, long long L,
                                int C) {
    grid_dep_sync();
    const int qn = C / 4;
    const int G = blockDim.x / qn;
    const int q = threadIdx.x % qn, g = threadIdx.x / qn;
    if (g >= G) return;
    const int c = q * 4;
    float4 wk[7];
#pragma unroll
    for (int k = 0; k < 7; ++k)
        wk[k] = make_float4(w[(c + 0) * 7 + k], w[(c + 1) * 7 + k], w[(c + 2) * 7 + k], w[(c + 3) * 7 + k]);
    const float4 bb = *reinterpret_cast<const float4*>(bias + c);
    const long long runs = (L + kHeadRun - 1) / kHeadRun;
    for (long long r = static_cast<long long>(blockIdx.x) * G + g; r < B * runs;
         r += static_cast<long long>(gridDim.x) * G) {
        const long long b = r / runs;
        const long long t0 = (r - b * runs) * kHeadRun;
        const long long t1 = min(t0 + kHeadRun, L);
        const float* a = audio + b * L;
        float win[7];  // samples t - 6 .. t
#pragma unroll
        for (int k = 0; k < 6; ++k) {
            const long long src = t0 + k - 6;
            win[k + 1] = src >= 0 ? __half2float(__float2half_rn(a[src])) : 0.f;
        }
        float* xo = x + (b * L + t0) * C + c;
        for (long long t = t0; t < t1; ++t, xo += C) {
#pragma unroll
            for (int k = 0; k < 6; ++k) win[k] = win[k + 1];
            win[6] = __half2float(__float2half_rn(a[t]));
            float4 acc = bb;
#pragma unroll
            for (int k = 0; k < 7; ++k) {
                acc.x = fmaf(wk[k].x, win[k], acc.x);
                acc.y = fmaf(wk[k].y, win[k], acc.y);
                acc.z = fmaf(wk[k].z, win[k], acc.z);
                acc.w = fmaf(wk[k].w, win[k], acc.w);
            }
            *reinterpret_cast<float4*>(xo) = acc;
        }
    }
}

// col[(b*Lout + t)][k*C + c] = g[b*L + t*s + k - lpad][c] (zero where that
// row is before the sequence start: the causal left padding): the im2col
// operand of a strided causal conv over the fp16 (already Snake-activated)
// input, in the column order k*C + c of the conv weight's [Cout][K][Cin]
// copy, so each output row is K whole input rows.  One 16-byte chunk (8
// channels) per thread; C % 8 == 0.
__global__ void im2col_rows_kernel(const __half* __restrict__ g, __half* __restrict__ col, int B, int L, int C, int K,
                                   int s, int lpad, int Lout) {
    grid_dep_sync();
    const int c8n = C / 8;
    const long long per_row = static_cast<long long>(K) * c8n;
    const long long total = static_cast<long long>(B) * Lout * per_row;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long n = i / per_row;
        const int rem = static_cast<int>(i - n * per_row);
        const int k = rem / c8n, c8 = rem - k * c8n;
        const int b = static_cast<int>(n / Lout);
        const int t = static_cast<int>(n - static_cast<long long>(b) * Lout);
        const int src = t * s + k - lpad;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (src >= 0 && src < L)
            v = *reinterpret_cast<const uint4*>(g + (static_cast<long long>(b) * L + src) * C + c8 * 8);
        reinterpret_cast<uint4*>(col)[i] = v;
    }
}

// out[(co*K + k)*Cin + ci] = in[(co*Cin + ci)*K + k]: a conv weight's
// [Cout][Cin][K] -> fp16 [Cout][K][Cin] (once, when the encoder is bound).
// `in` holds fp16 values, or Q4_0 blocks (in_q4) along that same element
// order, each value (q - 8) * d rounded once to fp16.
__global__ void permute_ck_kernel(const void* __restrict__ in, int in_q4, __half* __restrict__ out, int Cout,
                                  int Cin, int K) {
    const long long total = static_cast<long long>(Cout) * Cin * K;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int ci = static_cast<int>(i % Cin);
        const long long r = i / Cin;
        const int k = static_cast<int>(r % K);
        const long long co = r / K;
        const long long e = (co * Cin + ci) * K + k;
        if (in_q4) {
            const uint8_t* blk = static_cast<const uint8_t*>(in) + (e >> 5) * 18;
            const int j = static_cast<int>(e & 31);
            const float d = half_bits_to_float(static_cast<uint16_t>(blk[0] | (blk[1] << 8)));
            const int q = j < 16 ? (blk[2 + j] & 15) : (blk[2 + j - 16] >> 4);
            out[i] = __float2half_rn(static_cast<float>(q - 8) * d);
        } else {
            out[i] = static_cast<const __half*>(in)[e];
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
