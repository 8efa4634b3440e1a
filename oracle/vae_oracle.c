/*
 * vae_oracle.c -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * A plain-C restatement of the reference AudioVAE decoder (and encoder)
 * (nowang6/voxcpm-inference) used by tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py to check the CUDA path.  Nothing in the product
 * library links or calls this file.
 *
 * Pinned against the reference itself: tests/golden/ holds outputs of the
 * reference's own code (oracle/_ref, built from its sources by
 * oracle/Makefile.ref) on seeded models and latents, and
 * tests/test_oracle_golden.py checks this file against them.
 *
 * Activation layout everywhere: x[n][c], channels fastest ("L2 layout",
 * audio-vae.cpp:707-719), n = b*T + t.
 *
 * Numerics modes for the GEMM-like layers (pointwise, transposed conv, final
 * conv):
 *   VO_MODE_EXACT : fp32 activations, weights dequantised exactly to fp32.
 *   VO_MODE_REF   : the reference's L1 arithmetic.  ggml mul_mat rounds
 *                   activations to fp16 for F16 weights (vec_dot_type F16,
 *                   ggml-cpu.c:221-226) and quantises them to Q8_0 for Q4_0
 *                   weights (ggml-cpu.c:239-271, AVX2 quantize_row_q8_0 in
 *                   arch/x86/quants.c:302-360: d = amax/127, id = 127/amax,
 *                   round-half-even), dotting int blocks with fp32 scales
 *                   (ggml_vec_dot_q4_0_q8_0).  The F16 transposed conv rounds
 *                   its input to fp16 (ops.cpp:6155-6241); the Q4_0 one is
 *                   cast to F32 first (audio-vae.cpp:142-152) and runs in
 *                   fp32 (ops.cpp:6243-6350).  The final k7 conv goes through
 *                   im2col + F16 mul_mat (audio-vae.cpp:218-234), so its
 *                   input is rounded to fp16 too.
 *   VO_MODE_GPU   : the arithmetic the CUDA kernels use: every tensor-core
 *                   operand rounded to fp16 (activations, and Q4_0 weights
 *                   after exact dequantisation), fp32 accumulation; the final
 *                   conv's input rounded to fp16 as in VO_MODE_REF.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define VO_MODE_EXACT 0
#define VO_MODE_REF 1
#define VO_MODE_GPU 2

#define T_F32 0
#define T_F16 1
#define T_Q4_0 2
#define T_Q8_0 8

/* ---------------------------------------------------------------- fp16 --- */

/* IEEE binary16 -> binary32, exact. */
float vo_f16_to_f32(uint16_t h) {
    const uint32_t s = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1f;
    uint32_t m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = s;
        } else { /* subnormal: renormalise */
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; ++sh; }
            m &= 0x3ffu;
            bits = s | ((uint32_t)(127 - 15 + 1 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = s | 0x7f800000u | (m << 13);
    } else {
        bits = s | ((e + 127 - 15) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* binary32 -> binary16, round to nearest even (what F16C / ggml do). */
uint16_t vo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
    }
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* overflow -> inf */
    if (ax < 0x38800000u) {                                   /* subnormal / zero */
        if (ax < 0x33000000u) return (uint16_t)sign;
        const uint32_t e = ax >> 23;
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const int shift = (int)(126 - e); /* 14..24: units of 2^-24 */
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((ax >> 13) - (112u << 10));
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) ++q;
    return (uint16_t)(sign | q);
}

static inline float r16(float x) { return vo_f16_to_f32(vo_f32_to_f16(x)); }

/* ----------------------------------------------------------- Q4_0 / Q8_0 --
 * block_q4_0 = { fp16 d; uint8 qs[16] } (ggml-common.h:194-199), value
 * (nibble - 8) * d, low nibbles are elements 0..15, high nibbles 16..31. */

void vo_dequant_q4_0(const uint8_t* blocks, int64_t n, float* out) {
    for (int64_t b = 0; b < n / 32; ++b) {
        const uint8_t* blk = blocks + b * 18;
        const float d = vo_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        for (int j = 0; j < 16; ++j) {
            out[b * 32 + j] = (float)((blk[2 + j] & 0x0f) - 8) * d;
            out[b * 32 + 16 + j] = (float)((blk[2 + j] >> 4) - 8) * d;
        }
    }
}

/* ggml-quants.c:113-145 quantize_row_q4_0_ref. */
void vo_quantize_q4_0(const float* x, int64_t n, uint8_t* blocks) {
    for (int64_t b = 0; b < n / 32; ++b) {
        const float* v = x + b * 32;
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < 32; ++j) {
            if (amax < fabsf(v[j])) { amax = fabsf(v[j]); max = v[j]; }
        }
        const float d = max / -8;
        const float id = d ? 1.0f / d : 0.0f;
        const uint16_t h = vo_f32_to_f16(d);
        uint8_t* blk = blocks + b * 18;
        blk[0] = (uint8_t)(h & 0xff);
        blk[1] = (uint8_t)(h >> 8);
        for (int j = 0; j < 16; ++j) {
            const float x0 = v[j] * id, x1 = v[16 + j] * id;
            int8_t i0 = (int8_t)(x0 + 8.5f), i1 = (int8_t)(x1 + 8.5f);
            uint8_t q0 = (uint8_t)i0 > 15 ? 15 : (uint8_t)i0;
            uint8_t q1 = (uint8_t)i1 > 15 ? 15 : (uint8_t)i1;
            blk[2 + j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

/* Q8_0 activation quantisation as the AVX2 CPU backend does it. */
static void quantize_q8_0_avx2_semantics(const float* x, int64_t n, int8_t* q, float* d_out) {
    for (int64_t b = 0; b < n / 32; ++b) {
        const float* v = x + b * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
        const float d = amax / 127.f;
        const float id = amax != 0.0f ? 127.f / amax : 0.0f;
        d_out[b] = r16(d);
        for (int j = 0; j < 32; ++j) q[b * 32 + j] = (int8_t)nearbyintf(v[j] * id);
    }
}

/* ----------------------------------------------------------------- GGUF --- */

typedef struct {
    char name[96];
    int type;
    int n_dims;
    int64_t ne[4];
    uint64_t offset;
    const uint8_t* data;
} vo_tensor;

typedef struct {
    int latent_dim, decoder_dim, n_rates;
    int rates[8];
    int encoder_dim, n_enc_rates;
    int enc_rates[8];
    int n_tensors;
    vo_tensor* tensors;
    uint8_t* file;
    size_t file_size;
    /* derived fp32 weights, GEMM layout [M][K] */
    float* dw0;   /* [C][7] */
    float* pw1;   /* [1536][64] */
    float* convt[8];    /* [(co*2s + k)][ci] */
    float* res_pw[8][3];
    float* res_dw[8][3];
    float* fin;   /* [96][7] */
} vo_model;

static uint64_t rd_u64(const uint8_t** p) { uint64_t v; memcpy(&v, *p, 8); *p += 8; return v; }
static uint32_t rd_u32(const uint8_t** p) { uint32_t v; memcpy(&v, *p, 4); *p += 4; return v; }

static size_t gguf_scalar_size(uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: return 1;
        case 2: case 3: return 2;
        case 4: case 5: case 6: return 4;
        case 10: case 11: case 12: return 8;
        default: return 0;
    }
}

static void skip_value(const uint8_t** p, uint32_t t) {
    if (t == 8) { uint64_t n = rd_u64(p); *p += n; return; }
    if (t == 9) {
        uint32_t et = rd_u32(p);
        uint64_t n = rd_u64(p);
        for (uint64_t i = 0; i < n; ++i) skip_value(p, et);
        return;
    }
    *p += gguf_scalar_size(t);
}

static const vo_tensor* find(const vo_model* m, const char* name) {
    for (int i = 0; i < m->n_tensors; ++i)
        if (strcmp(m->tensors[i].name, name) == 0) return &m->tensors[i];
    return NULL;
}

static int64_t nelem(const vo_tensor* t) {
    int64_t n = 1;
    for (int i = 0; i < t->n_dims; ++i) n *= t->ne[i];
    return n;
}

/* Any F32/F16/Q4_0/Q8_0 tensor to fp32 in its memory order. */
static float* to_f32(const vo_tensor* t) {
    const int64_t n = nelem(t);
    float* o = (float*)malloc(sizeof(float) * (size_t)n);
    if (t->type == T_F32) {
        memcpy(o, t->data, sizeof(float) * (size_t)n);
    } else if (t->type == T_F16) {
        for (int64_t i = 0; i < n; ++i) {
            uint16_t h;
            memcpy(&h, t->data + 2 * i, 2);
            o[i] = vo_f16_to_f32(h);
        }
    } else if (t->type == T_Q4_0) {
        vo_dequant_q4_0(t->data, n, o);
    } else if (t->type == T_Q8_0) {
        for (int64_t b = 0; b < n / 32; ++b) {
            const uint8_t* blk = t->data + b * 34;
            const float d = vo_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            for (int j = 0; j < 32; ++j) o[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
        }
    } else {
        free(o);
        return NULL;
    }
    return o;
}

static const vo_tensor* need(const vo_model* m, const char* name) {
    const vo_tensor* t = find(m, name);
    if (!t) fprintf(stderr, "vae_oracle: missing tensor %s\n", name);
    return t;
}

void vo_close(vo_model* m);

vo_model* vo_open(const char* path) {
    FILE* f = fopen(path, "rb");
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    const size_t sz = (size_t)ftell(f);
    fseek(f, 0, SEEK_SET);
    vo_model* m = (vo_model*)calloc(1, sizeof(vo_model));
    m->file = (uint8_t*)malloc(sz);
    m->file_size = sz;
    if (fread(m->file, 1, sz, f) != sz) { fclose(f); vo_close(m); return NULL; }
    fclose(f);
    const uint8_t* p = m->file;
    if (memcmp(p, "GGUF", 4) != 0) { vo_close(m); return NULL; }
    p += 4;
    rd_u32(&p); /* version */
    const uint64_t n_t = rd_u64(&p), n_kv = rd_u64(&p);
    uint32_t alignment = 32;
    m->latent_dim = 64;
    m->decoder_dim = 1536;
    for (uint64_t i = 0; i < n_kv; ++i) {
        const uint64_t kl = rd_u64(&p);
        char key[256] = {0};
        memcpy(key, p, kl < 255 ? kl : 255);
        p += kl;
        const uint32_t t = rd_u32(&p);
        if (!strcmp(key, "voxcpm_audio_vae_config_latent_dim") && t == 4) {
            m->latent_dim = (int)rd_u32(&p);
        } else if (!strcmp(key, "voxcpm_audio_vae_config_decoder_dim") && t == 4) {
            m->decoder_dim = (int)rd_u32(&p);
        } else if (!strcmp(key, "voxcpm_audio_vae_config_encoder_dim") && t == 4) {
            m->encoder_dim = (int)rd_u32(&p);
        } else if (!strcmp(key, "voxcpm_audio_vae_config_encoder_rates") && t == 9) {
            const uint32_t et = rd_u32(&p);
            const uint64_t n = rd_u64(&p);
            m->n_enc_rates = (int)n;
            for (uint64_t j = 0; j < n; ++j) {
                if (et == 5 || et == 4) m->enc_rates[j] = (int)rd_u32(&p);
                else skip_value(&p, et);
            }
        } else if (!strcmp(key, "general.alignment") && t == 4) {
            alignment = rd_u32(&p);
        } else if (!strcmp(key, "voxcpm_audio_vae_config_decoder_rates") && t == 9) {
            const uint32_t et = rd_u32(&p);
            const uint64_t n = rd_u64(&p);
            m->n_rates = (int)n;
            for (uint64_t j = 0; j < n; ++j) {
                if (et == 5 || et == 4) m->rates[j] = (int)rd_u32(&p);
                else skip_value(&p, et);
            }
        } else {
            skip_value(&p, t);
        }
    }
    m->n_tensors = (int)n_t;
    m->tensors = (vo_tensor*)calloc(n_t, sizeof(vo_tensor));
    for (uint64_t i = 0; i < n_t; ++i) {
        vo_tensor* t = &m->tensors[i];
        const uint64_t nl = rd_u64(&p);
        memcpy(t->name, p, nl < 95 ? nl : 95);
        p += nl;
        t->n_dims = (int)rd_u32(&p);
        for (int d = 0; d < 4; ++d) t->ne[d] = 1;
        for (int d = 0; d < t->n_dims; ++d) t->ne[d] = (int64_t)rd_u64(&p);
        t->type = (int)rd_u32(&p);
        t->offset = rd_u64(&p);
    }
    size_t off = (size_t)(p - m->file);
    off = (off + alignment - 1) / alignment * alignment;
    for (uint64_t i = 0; i < n_t; ++i) m->tensors[i].data = m->file + off + m->tensors[i].offset;

    /* derived fp32 weights */
    char nm[256];
    const char* pre = "audio_vae.decoder.model.";
    snprintf(nm, sizeof nm, "%s0.weight", pre);
    const vo_tensor* t = need(m, nm);
    if (!t) { vo_close(m); return NULL; }
    m->dw0 = to_f32(t); /* [C][7] memory order already (ne = [7,1,C]) */
    snprintf(nm, sizeof nm, "%s1.weight", pre);
    if (!(t = need(m, nm))) { vo_close(m); return NULL; }
    m->pw1 = to_f32(t); /* [Cout][Cin] */
    int C = m->decoder_dim;
    for (int b = 0; b < m->n_rates; ++b) {
        const int s = m->rates[b], co = C / 2, K = 2 * s;
        snprintf(nm, sizeof nm, "%s%d.block.1.weight", pre, b + 2);
        if (!(t = need(m, nm))) { vo_close(m); return NULL; }
        float* raw = to_f32(t); /* raw[ci][co*K + k] */
        float* w = (float*)malloc(sizeof(float) * (size_t)K * co * C);
        for (int ci = 0; ci < C; ++ci)
            for (int j = 0; j < K * co; ++j) w[(size_t)j * C + ci] = raw[(size_t)ci * K * co + j];
        free(raw);
        m->convt[b] = w; /* [co*K + k][ci] */
        for (int r = 0; r < 3; ++r) {
            snprintf(nm, sizeof nm, "%s%d.block.%d.block.1.weight", pre, b + 2, r + 2);
            if (!(t = need(m, nm))) { vo_close(m); return NULL; }
            m->res_dw[b][r] = to_f32(t);
            snprintf(nm, sizeof nm, "%s%d.block.%d.block.3.weight", pre, b + 2, r + 2);
            if (!(t = need(m, nm))) { vo_close(m); return NULL; }
            m->res_pw[b][r] = to_f32(t);
        }
        C = co;
    }
    snprintf(nm, sizeof nm, "%s%d.weight", pre, m->n_rates + 3);
    if (!(t = need(m, nm))) { vo_close(m); return NULL; }
    m->fin = to_f32(t); /* ne [7, C, 1] -> [c][k] */
    return m;
}

void vo_close(vo_model* m) {
    if (!m) return;
    free(m->dw0);
    free(m->pw1);
    for (int b = 0; b < 8; ++b) {
        free(m->convt[b]);
        for (int r = 0; r < 3; ++r) { free(m->res_pw[b][r]); free(m->res_dw[b][r]); }
    }
    free(m->fin);
    free(m->tensors);
    free(m->file);
    free(m);
}

int vo_num_blocks(const vo_model* m) { return m->n_rates; }
int vo_rate(const vo_model* m, int b) { return m->rates[b]; }
int vo_decoder_dim(const vo_model* m) { return m->decoder_dim; }
int vo_latent_dim(const vo_model* m) { return m->latent_dim; }

static float* vec_f32(const vo_model* m, const char* name) {
    const vo_tensor* t = need(m, name);
    return t ? to_f32(t) : NULL;
}

/* ------------------------------------------------------------ the ops --- */

/* snake (audio-vae.cpp:278-289 L1, :1443-1479 L2):
 * y = x + sin(a*x)^2 * (1 / (a + 1e-9)), per channel a; libm sinf as ggml_sin. */
void vo_snake(const float* x, const float* alpha, int C, int64_t N, float* y) {
    for (int64_t n = 0; n < N; ++n)
        for (int c = 0; c < C; ++c) {
            const float v = x[n * C + c];
            const float s = sinf(alpha[c] * v);
            y[n * C + c] = v + (s * s) * (1.0f / (alpha[c] + 1e-9f));
        }
}

/* depthwise causal conv (audio-vae.cpp:157-214 / :1074-1205):
 * y[t][c] = b[c] + sum_k x[t + k*d - 6d][c] * w[c][k], zero before t=0;
 * sequences of T samples are independent (B = N / T). */
void vo_dwconv(const float* x, const float* w /*[C][7]*/, const float* b, int C, int T, int B,
               int d, float* y) {
    for (int bb = 0; bb < B; ++bb)
        for (int t = 0; t < T; ++t)
            for (int c = 0; c < C; ++c) {
                float acc = b ? b[c] : 0.0f;
                for (int k = 0; k < 7; ++k) {
                    const int st = t + k * d - 6 * d;
                    if (st < 0 || st >= T) continue;
                    /* the reference's scalar loop `sum += x * w` is contracted to
                     * an FMA by GCC on FMA-capable x86 builds */
                    acc = fmaf(x[((int64_t)bb * T + st) * C + c], w[c * 7 + k], acc);
                }
                y[((int64_t)bb * T + t) * C + c] = acc;
            }
}

/* Rounds (GPU/REF-F16 modes) or block-quantises (REF-Q4_0 mode) a GEMM input. */
static float* prep_act(const float* x, int64_t N, int K, int wtype, int mode, int is_q8,
                       float** q8d_out) {
    float* xa = (float*)malloc(sizeof(float) * (size_t)N * K);
    if (mode == VO_MODE_REF && wtype == T_Q4_0 && is_q8) {
        int8_t* q = (int8_t*)malloc((size_t)N * K);
        float* d = (float*)malloc(sizeof(float) * (size_t)N * K / 32);
        for (int64_t n = 0; n < N; ++n) quantize_q8_0_avx2_semantics(x + n * K, K, q + n * K, d + n * K / 32);
        for (int64_t i = 0; i < N * K; ++i) xa[i] = (float)q[i];
        free(q);
        *q8d_out = d;
        return xa;
    }
    const int round16 = (mode == VO_MODE_GPU) || (mode == VO_MODE_REF && wtype == T_F16);
    for (int64_t i = 0; i < N * K; ++i) xa[i] = round16 ? r16(x[i]) : x[i];
    *q8d_out = NULL;
    return xa;
}

/* Weight preparation per mode: GPU mode rounds every weight to fp16. */
static float* prep_w(const float* w, int64_t n, int mode) {
    float* o = (float*)malloc(sizeof(float) * (size_t)n);
    for (int64_t i = 0; i < n; ++i) o[i] = mode == VO_MODE_GPU ? r16(w[i]) : w[i];
    return o;
}

/* pointwise conv + bias (+ residual): y[n][m] = b[m] + sum_k W[m][k] x[n][k] (+ r[n][m]).
 * raw_q4 (optional) are the Q4_0 blocks of W (row m = K/32 blocks), used by the
 * REF mode's int-dot emulation of ggml_vec_dot_q4_0_q8_0. */
void vo_pointwise(const float* W, const uint8_t* raw_q4, int wtype, const float* b, const float* res,
                  const float* x, int64_t N, int K, int M, int mode, float* y) {
    float* q8d = NULL;
    float* xa = prep_act(x, N, K, wtype, mode, 1, &q8d);
    if (q8d) {
        for (int64_t n = 0; n < N; ++n)
            for (int m = 0; m < M; ++m) {
                float acc = 0.0f;
                for (int kb = 0; kb < K / 32; ++kb) {
                    const uint8_t* blk = raw_q4 + ((size_t)m * (K / 32) + kb) * 18;
                    const float d4 = vo_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
                    int isum = 0;
                    for (int j = 0; j < 16; ++j) {
                        isum += ((blk[2 + j] & 0x0f) - 8) * (int)xa[n * K + kb * 32 + j];
                        isum += ((blk[2 + j] >> 4) - 8) * (int)xa[n * K + kb * 32 + 16 + j];
                    }
                    acc += (float)isum * (d4 * q8d[n * (K / 32) + kb]);
                }
                y[n * M + m] = acc + (b ? b[m] : 0.0f) + (res ? res[n * M + m] : 0.0f);
            }
        free(q8d);
    } else {
        float* wa = prep_w(W, (int64_t)M * K, mode);
        for (int64_t n = 0; n < N; ++n)
            for (int m = 0; m < M; ++m) {
                const float* wr = wa + (size_t)m * K;
                const float* xr = xa + n * K;
                double acc = 0.0;
                for (int k = 0; k < K; ++k) acc += (double)wr[k] * xr[k];
                y[n * M + m] = (float)acc + (b ? b[m] : 0.0f) + (res ? res[n * M + m] : 0.0f);
            }
        free(wa);
    }
    free(xa);
}

/* causal transposed conv, kernel 2s, stride s, cropped to T*s
 * (audio-vae.cpp:512-534, :1642-1673; ops.cpp:6155-6350):
 * y[t*s + r][co] = b[co] + sum_ci W[co*2s + r][ci] x[t][ci] + W[co*2s + s + r][ci] x[t-1][ci],
 * the second term absent at t = 0 of each sequence. */
void vo_convt(const float* W /*[co*2s+k][ci]*/, int wtype, int w_ndims, const float* b, const float* x,
              int T, int B, int Cin, int Cout, int s, int mode, float* y) {
    const int K = 2 * s;
    float* q8d = NULL;
    /* unfold_transpose_conv1d_weight (audio-vae.cpp:142-152) casts every folded
     * 2-D weight (Q4_0 or F16) to F32, so only a 3-D F16 weight reaches the
     * fp16-rounding kernel conv_transpose_1d_f16_f32. */
    const int eff_type = (wtype == T_F16 && w_ndims == 3) ? T_F16 : T_F32;
    float* xa = prep_act(x, (int64_t)B * T, Cin, eff_type, mode, 0, &q8d);
    float* wa = prep_w(W, (int64_t)K * Cout * Cin, mode);
    for (int bb = 0; bb < B; ++bb)
        for (int t = 0; t < T; ++t)
            for (int r = 0; r < s; ++r)
                for (int co = 0; co < Cout; ++co) {
                    double acc = 0.0;
                    const float* xr = xa + ((int64_t)bb * T + t) * Cin;
                    const float* wr = wa + ((size_t)co * K + r) * Cin;
                    for (int ci = 0; ci < Cin; ++ci) acc += (double)wr[ci] * xr[ci];
                    if (t > 0) {
                        const float* xp = xa + ((int64_t)bb * T + t - 1) * Cin;
                        const float* wp = wa + ((size_t)co * K + s + r) * Cin;
                        for (int ci = 0; ci < Cin; ++ci) acc += (double)wp[ci] * xp[ci];
                    }
                    y[(((int64_t)bb * T + t) * s + r) * Cout + co] = (float)acc + b[co];
                }
    free(xa);
    free(wa);
}

/* final causal conv k7 C->1 + tanh (audio-vae.cpp:1304-1392, :1631-1632):
 * y[t] = tanh(b + sum_c sum_k w[c][k] x[t + k - 6][c]). */
void vo_final(const float* x, const float* w /*[C][7]*/, float bias, int C, int T, int B, int mode,
              float* y) {
    for (int bb = 0; bb < B; ++bb)
        for (int t = 0; t < T; ++t) {
            double acc = 0.0;
            for (int k = 0; k < 7; ++k) {
                const int st = t + k - 6;
                if (st < 0) continue;
                const float* xr = x + ((int64_t)bb * T + st) * C;
                for (int c = 0; c < C; ++c) {
                    const float v = mode == VO_MODE_EXACT ? xr[c] : r16(xr[c]);
                    acc += (double)w[c * 7 + k] * v;
                }
            }
            y[(int64_t)bb * T + t] = tanhf((float)acc + bias);
        }
}

/* ------------------------------------------------------------ decoder --- */

/* Full decode of B independent latents z[b][c][t] (ggml ne=[T,64] each) into
 * out[b][T*prod(rates)].  If stage >= 0, the activation after that stage is
 * copied to stage_out instead (stage numbering: 0 = model.0 dw, 1 = model.1
 * pw, then per block b: 2+4b convT, 3+4b..5+4b residual units; the final
 * stage is the waveform).  Returns the number of floats written. */
int64_t vo_decode(const vo_model* m, const float* z, int T, int B, int mode, int stage, float* out) {
    char nm[256];
    const char* pre = "audio_vae.decoder.model.";
    const int L = m->latent_dim;
    int64_t N = (int64_t)B * T;
    int C = L;
    int Tc = T;
    float* x = (float*)malloc(sizeof(float) * (size_t)N * L);
    for (int bb = 0; bb < B; ++bb)
        for (int c = 0; c < L; ++c)
            for (int t = 0; t < T; ++t)
                x[((int64_t)bb * T + t) * L + c] = z[((int64_t)bb * L + c) * T + t];
    int cur = 0;
#define STAGE_DONE(buf, count)                                     \
    do {                                                           \
        if (stage == cur) {                                        \
            memcpy(out, buf, sizeof(float) * (size_t)(count));     \
            free(buf);                                             \
            return (count);                                        \
        }                                                          \
        ++cur;                                                     \
    } while (0)

    /* model.0: dw k7, causal pad 6 */
    snprintf(nm, sizeof nm, "%s0.bias", pre);
    float* b0 = vec_f32(m, nm);
    float* y = (float*)malloc(sizeof(float) * (size_t)N * C);
    vo_dwconv(x, m->dw0, b0, C, Tc, B, 1, y);
    free(b0);
    free(x);
    x = y;
    STAGE_DONE(x, N * C);

    /* model.1: pw latent -> decoder_dim */
    snprintf(nm, sizeof nm, "%s1.weight", pre);
    const vo_tensor* w1 = find(m, nm);
    snprintf(nm, sizeof nm, "%s1.bias", pre);
    float* b1 = vec_f32(m, nm);
    const int D = m->decoder_dim;
    y = (float*)malloc(sizeof(float) * (size_t)N * D);
    vo_pointwise(m->pw1, w1->data, w1->type, b1, NULL, x, N, C, D, mode, y);
    free(b1);
    free(x);
    x = y;
    C = D;
    STAGE_DONE(x, N * C);

    for (int bi = 0; bi < m->n_rates; ++bi) {
        const int s = m->rates[bi], co = C / 2;
        snprintf(nm, sizeof nm, "%s%d.block.0.alpha", pre, bi + 2);
        float* a = vec_f32(m, nm);
        float* h = (float*)malloc(sizeof(float) * (size_t)N * C);
        vo_snake(x, a, C, N, h);
        free(a);
        snprintf(nm, sizeof nm, "%s%d.block.1.weight", pre, bi + 2);
        const vo_tensor* wt = find(m, nm);
        snprintf(nm, sizeof nm, "%s%d.block.1.bias", pre, bi + 2);
        float* bt = vec_f32(m, nm);
        float* yc = (float*)malloc(sizeof(float) * (size_t)N * s * co);
        vo_convt(m->convt[bi], wt->type, wt->n_dims, bt, h, Tc, B, C, co, s, mode, yc);
        free(bt);
        free(h);
        free(x);
        x = yc;
        N *= s;
        Tc *= s;
        C = co;
        STAGE_DONE(x, N * C);
        const int dil[3] = {1, 3, 9};
        for (int r = 0; r < 3; ++r) {
            char rp[128];
            snprintf(rp, sizeof rp, "%s%d.block.%d.block.", pre, bi + 2, r + 2);
            snprintf(nm, sizeof nm, "%s0.alpha", rp);
            float* a1 = vec_f32(m, nm);
            snprintf(nm, sizeof nm, "%s1.bias", rp);
            float* db = vec_f32(m, nm);
            snprintf(nm, sizeof nm, "%s2.alpha", rp);
            float* a2 = vec_f32(m, nm);
            snprintf(nm, sizeof nm, "%s3.weight", rp);
            const vo_tensor* pw = find(m, nm);
            snprintf(nm, sizeof nm, "%s3.bias", rp);
            float* pb = vec_f32(m, nm);
            float* h1 = (float*)malloc(sizeof(float) * (size_t)N * C);
            float* h2 = (float*)malloc(sizeof(float) * (size_t)N * C);
            vo_snake(x, a1, C, N, h1);
            vo_dwconv(h1, m->res_dw[bi][r], db, C, Tc, B, dil[r], h2);
            vo_snake(h2, a2, C, N, h1);
            float* yr = (float*)malloc(sizeof(float) * (size_t)N * C);
            vo_pointwise(m->res_pw[bi][r], pw->data, pw->type, pb, x, h1, N, C, C, mode, yr);
            free(h1);
            free(h2);
            free(a1);
            free(a2);
            free(db);
            free(pb);
            free(x);
            x = yr;
            STAGE_DONE(x, N * C);
        }
    }
    snprintf(nm, sizeof nm, "%s%d.alpha", pre, m->n_rates + 2);
    float* af = vec_f32(m, nm);
    float* h = (float*)malloc(sizeof(float) * (size_t)N * C);
    vo_snake(x, af, C, N, h);
    free(af);
    free(x);
    snprintf(nm, sizeof nm, "%s%d.bias", pre, m->n_rates + 3);
    float* bf = vec_f32(m, nm);
    vo_final(h, m->fin, bf[0], C, Tc, B, mode, out);
    free(bf);
    free(h);
    (void)cur;
    return N;
#undef STAGE_DONE
}

/* ------------------------------------------------------------ encoder --- */

/* Causal conv1d as the reference runs it (causal_conv1d, audio-vae.cpp:476-493:
 * left pad 2*padding = lpad, then im2col + mul_mat, :218-234): kernel K,
 * stride s, weight [Cout][Cin*K] in memory (row j = ci*K + k, the F16
 * [K, Cin, Cout] tensor or the folded Q4_0 [K*Cin, Cout]); x [B*Lin][Cin]
 * -> y [B*Lout][Cout], Lout = (Lin + lpad - K)/s + 1.  The im2col row is the
 * GEMM input, so the numerics modes apply to it as to a pointwise conv. */
static int64_t conv1d_k(const vo_tensor* wt, const float* b, const float* x, int64_t Lin, int B, int Cin,
                        int Cout, int K, int s, int lpad, int mode, float* y) {
    const int64_t Lout = (Lin + lpad - K) / s + 1;
    const int KC = K * Cin;
    float* col = (float*)calloc((size_t)B * Lout * KC, sizeof(float));
    for (int bb = 0; bb < B; ++bb)
        for (int64_t t = 0; t < Lout; ++t)
            for (int ci = 0; ci < Cin; ++ci)
                for (int k = 0; k < K; ++k) {
                    const int64_t src = t * s + k - lpad;
                    if (src < 0 || src >= Lin) continue;
                    col[((int64_t)bb * Lout + t) * KC + (int64_t)ci * K + k] = x[((int64_t)bb * Lin + src) * Cin + ci];
                }
    float* W = to_f32(wt);
    vo_pointwise(W, wt->data, wt->type, b, NULL, col, (int64_t)B * Lout, KC, Cout, mode, y);
    free(W);
    free(col);
    return Lout;
}

int vo_encoder_dim(const vo_model* m) { return m->encoder_dim; }
int vo_encoder_hop(const vo_model* m) {
    int h = 1;
    for (int i = 0; i < m->n_enc_rates; ++i) h *= m->enc_rates[i];
    return h;
}

/* Full encode of B waveforms audio[b][n] (AudioVAE::encode / encode_tensor,
 * audio-vae.cpp:640-664): zero-padded to a multiple of the hop (preprocess,
 * :465-474), head conv k7 (pad 3) -> per block three residual units (d = 1,
 * 3, 9), Snake, conv k 2s stride s (pad ceil(s/2)) doubling the channels
 * (encoder_block_forward, :553-570) -> fc_mu conv k3 (pad 1).  The latent goes
 * to out[b][c][t] (ggml ne=[T, latent] per waveform).  Returns T, or -1 when
 * the model holds no encoder (placeholder tensors). */
int64_t vo_encode_stage(const vo_model* m, const float* audio, int64_t n, int B, int mode, int stage, float* out);
int64_t vo_encode(const vo_model* m, const float* audio, int64_t n, int B, int mode, float* out) {
    return vo_encode_stage(m, audio, n, B, mode, -1, out);
}

/* As vo_encode; stage >= 0 stops after that stage (0 = head conv, then per
 * block b: 1+4b..3+4b the residual units, 4+4b the Snake + strided conv) and
 * copies its activation [B*L][C] to out, returning the element count. */
int64_t vo_encode_stage(const vo_model* m, const float* audio, int64_t n, int B, int mode, int stage, float* out) {
    int cur = 0;
#define ENC_STAGE(buf, count)                                  \
    do {                                                       \
        if (stage == cur) {                                    \
            memcpy(out, buf, sizeof(float) * (size_t)(count)); \
            free(buf);                                         \
            return (count);                                    \
        }                                                      \
        ++cur;                                                 \
    } while (0)
    char nm[256];
    const char* pre = "audio_vae.encoder.";
    const int E = m->encoder_dim, hop = vo_encoder_hop(m);
    snprintf(nm, sizeof nm, "%sblock.0.weight", pre);
    const vo_tensor* w0 = find(m, nm);
    if (!w0 || E <= 0 || nelem(w0) != 7 * (int64_t)E || m->n_enc_rates <= 0) return -1;
    const int64_t Lp = (n + hop - 1) / hop * hop;
    float* x = (float*)calloc((size_t)B * Lp, sizeof(float));
    for (int bb = 0; bb < B; ++bb) memcpy(x + (int64_t)bb * Lp, audio + (int64_t)bb * n, sizeof(float) * (size_t)n);
    int64_t L = Lp;
    int C = E;
    snprintf(nm, sizeof nm, "%sblock.0.bias", pre);
    float* b0 = vec_f32(m, nm);
    float* y = (float*)malloc(sizeof(float) * (size_t)B * L * C);
    conv1d_k(w0, b0, x, L, B, 1, C, 7, 1, 6, mode, y);
    free(b0);
    free(x);
    x = y;
    ENC_STAGE(x, (int64_t)B * L * C);
    const int dil[3] = {1, 3, 9};
    for (int bi = 0; bi < m->n_enc_rates; ++bi) {
        const int s = m->enc_rates[bi];
        const int64_t N = (int64_t)B * L;
        for (int r = 0; r < 3; ++r) {
            char rp[128];
            snprintf(rp, sizeof rp, "%sblock.%d.block.%d.block.", pre, bi + 1, r);
            snprintf(nm, sizeof nm, "%s0.alpha", rp);
            float* a1 = vec_f32(m, nm);
            snprintf(nm, sizeof nm, "%s1.weight", rp);
            float* dw = vec_f32(m, nm);
            snprintf(nm, sizeof nm, "%s1.bias", rp);
            float* db = vec_f32(m, nm);
            snprintf(nm, sizeof nm, "%s2.alpha", rp);
            float* a2 = vec_f32(m, nm);
            snprintf(nm, sizeof nm, "%s3.weight", rp);
            const vo_tensor* pw = find(m, nm);
            snprintf(nm, sizeof nm, "%s3.bias", rp);
            float* pb = vec_f32(m, nm);
            float* W = to_f32(pw);
            float* h1 = (float*)malloc(sizeof(float) * (size_t)N * C);
            float* h2 = (float*)malloc(sizeof(float) * (size_t)N * C);
            vo_snake(x, a1, C, N, h1);
            vo_dwconv(h1, dw, db, C, (int)L, B, dil[r], h2);
            vo_snake(h2, a2, C, N, h1);
            float* yr = (float*)malloc(sizeof(float) * (size_t)N * C);
            vo_pointwise(W, pw->data, pw->type, pb, x, h1, N, C, C, mode, yr);
            free(W);
            free(h1);
            free(h2);
            free(a1);
            free(dw);
            free(db);
            free(a2);
            free(pb);
            free(x);
            x = yr;
            ENC_STAGE(x, N * C);
        }
        snprintf(nm, sizeof nm, "%sblock.%d.block.3.alpha", pre, bi + 1);
        float* a = vec_f32(m, nm);
        float* h = (float*)malloc(sizeof(float) * (size_t)N * C);
        vo_snake(x, a, C, N, h);
        free(a);
        free(x);
        snprintf(nm, sizeof nm, "%sblock.%d.block.4.weight", pre, bi + 1);
        const vo_tensor* wc = find(m, nm);
        snprintf(nm, sizeof nm, "%sblock.%d.block.4.bias", pre, bi + 1);
        float* bc = vec_f32(m, nm);
        const int64_t Lo = (L + 2 * ((s + 1) / 2) - 2 * s) / s + 1;
        y = (float*)malloc(sizeof(float) * (size_t)B * Lo * 2 * C);
        conv1d_k(wc, bc, h, L, B, C, 2 * C, 2 * s, s, 2 * ((s + 1) / 2), mode, y);
        free(bc);
        free(h);
        x = y;
        L = Lo;
        C *= 2;
        ENC_STAGE(x, (int64_t)B * L * C);
    }
    const int Lt = m->latent_dim;
    snprintf(nm, sizeof nm, "%sfc_mu.weight", pre);
    const vo_tensor* wf = find(m, nm);
    snprintf(nm, sizeof nm, "%sfc_mu.bias", pre);
    float* bf = vec_f32(m, nm);
    y = (float*)malloc(sizeof(float) * (size_t)B * L * Lt);
    conv1d_k(wf, bf, x, L, B, C, Lt, 3, 1, 2, mode, y);
    free(bf);
    free(x);
    for (int bb = 0; bb < B; ++bb)
        for (int c = 0; c < Lt; ++c)
            for (int64_t t = 0; t < L; ++t) out[((int64_t)bb * Lt + c) * L + t] = y[((int64_t)bb * L + t) * Lt + c];
    free(y);
    (void)cur;
    return L;
#undef ENC_STAGE
}
