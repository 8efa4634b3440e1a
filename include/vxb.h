/*
 * vxb.h -- C ABI of the B200 AudioVAE decoder and encoder (libvxb.so).
 *
 * This is the drop-in seam for the reference's decode path
 * (nowang6/voxcpm-inference): plain pointers, sizes and int status codes; no
 * C++ types and no exceptions cross it.  Each entry point names the reference
 * interface it replaces (reference file:line).  Device pointers are CUDA
 * global-memory addresses on the context's device; host pointers are
 * ordinary (preferably pinned) host memory.
 *
 * Threading: one vxb_ctx per GPU per host thread; calls on one context are
 * not thread-safe.  Every function returns VXB_OK (0) or a VXB_ERR_* code;
 * vxb_last_error() gives the calling thread's last message.
 */
#ifndef VXB_H
#define VXB_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VXB_API __attribute__((visibility("default")))
#else
#define VXB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes; the non-zero ones map onto voxcpm::ErrorCode
 * (reference include/voxcpm/common.h:69-79). */
#define VXB_OK 0
#define VXB_ERR_INVALID_ARGUMENT 1
#define VXB_ERR_OUT_OF_MEMORY 2
#define VXB_ERR_FILE_NOT_FOUND 3
#define VXB_ERR_INVALID_FORMAT 4
#define VXB_ERR_BACKEND 5        /* CUDA error */
#define VXB_ERR_NOT_READY 6      /* weights / plan missing (reference asserts instead) */
#define VXB_ERR_TIMEOUT 7        /* bounded host wait expired */
#define VXB_ERR_DEVICE_STATUS 8  /* a kernel's bounded device wait gave up */
#define VXB_ERR_MISSING_TENSOR 9 /* required tensor absent (load_from_store -> false) */

/* ggml tensor types accepted by vxb_upload_tensor (ggml.h enum values). */
#define VXB_TYPE_F32 0
#define VXB_TYPE_F16 1
#define VXB_TYPE_Q4_0 2

typedef struct vxb_ctx vxb_ctx;

/* Last error message of the calling thread ("" if none). */
VXB_API const char* vxb_last_error(void);

/* Creates a context on CUDA device `device` with its own stream.
 * Replaces VoxCPMBackend::VoxCPMBackend(BackendType, int) (include/voxcpm/backend.h:53,
 * src/backend.cpp:91-121), which throws voxcpm::Error on init failure. */
VXB_API int vxb_open(int device, vxb_ctx** out);

/* Frees every device and host resource of the context (weights, plan, graph).
 * Replaces ~VoxCPMBackend / ~VoxCPMWeightStore / ~AudioVAE
 * (src/weight-store.cpp:55-76, src/audio-vae.cpp:295-329). */
VXB_API int vxb_close(vxb_ctx* ctx);

/* Decoder hyper-parameters, as AudioVAE::load_from_store reads them from the
 * GGUF KV voxcpm_audio_vae_config_{latent_dim,decoder_dim,decoder_rates}
 * (src/audio-vae.cpp:421-463, include/voxcpm/config.h:34-133). */
VXB_API int vxb_set_config(vxb_ctx* ctx, int latent_dim, int decoder_dim, const int* rates, int n_rates);

/* Uploads one tensor's bytes unchanged (F32, F16 or Q4_0 blocks) to HBM under
 * its GGUF name; ne/n_dims are ggml's (ne[0] fastest).  Replaces the per-tensor
 * fread into the backend buffer in VoxCPMWeightStore::load_from_file
 * (src/weight-store.cpp:13-51, :78-225). */
VXB_API int vxb_upload_tensor(vxb_ctx* ctx, const char* name, int ggml_type, const int64_t* ne, int n_dims,
                      const void* host_data, size_t nbytes);

/* Parses a GGUF file, applies its decoder config and uploads every tensor.
 * Replaces VoxCPMWeightStore::load_from_file + the KV part of
 * AudioVAE::load_from_store (src/weight-store.cpp:78-225, src/audio-vae.cpp:421-463).
 * Missing required KV keys -> VXB_ERR_INVALID_FORMAT. */
VXB_API int vxb_load_gguf(vxb_ctx* ctx, const char* path);

/* Binds the decoder tensors by name, checks their shapes and builds the
 * derived fp32 vectors (bias, Snake alpha, inv = 1/(alpha+1e-9), depthwise
 * taps) on the device.  Idempotent.  Replaces load_decoder_weights +
 * AudioVAE::ensure_derived_weights (src/audio-vae.cpp:365-419, :839-1003);
 * a missing tensor gives VXB_ERR_MISSING_TENSOR, as load_from_store returns
 * false.  Unlike the reference (which asserts Q4_0 convT weights at :739),
 * F16 (2-D folded or 3-D) and Q4_0 are both accepted.
 * Q4_0 conv weights stay Q4_0: besides the uploaded blocks, prepare lays the
 * same nibbles and scales out once as 16-byte aligned rows (the same 4.5
 * bits per value; +15.1 MB of HBM for the VoxCPM decoder), which the plan's
 * GEMMs load by TMA and dequantise to fp16 in shared memory inside their
 * mainloop; the fused residual-unit kernels dequantise the uploaded blocks
 * once per CTA.  With vxb_set_q4_fp16_cache(ctx, 1) prepare instead makes an
 * fp16 copy of each Q4_0 conv weight (+53.7 MB for the VoxCPM decoder) that the GEMMs
 * read directly: the same operand values and results, traded for HBM. */
VXB_API int vxb_prepare(vxb_ctx* ctx);

/* Opt-in (enable != 0) or out of the fp16 copies of Q4_0 conv weights that
 * vxb_prepare makes for the decode and encode plans' GEMMs (see vxb_prepare);
 * takes effect at the next vxb_prepare.  Off by default.  No counterpart in
 * the reference, whose CPU path dots Q4_0 blocks directly. */
VXB_API int vxb_set_q4_fp16_cache(vxb_ctx* ctx, int enable);

/* Allocates the activation arena for `batch` independent latents of `T` frames
 * and captures the whole decode as one CUDA graph (use_graph != 0) or keeps
 * it as a launch list.  Replaces the per-step graph build + gallocr reserve
 * in AudioVAE::decode / VoxCPMBackend::reserve_compute_memory / alloc_graph
 * (src/audio-vae.cpp:666-700, src/backend.cpp:241-287). */
VXB_API int vxb_build_plan(vxb_ctx* ctx, int batch, int T, int use_graph);

/* Samples per latent frame (product of the decoder rates, 640 for VoxCPM). */
VXB_API int vxb_hop(const vxb_ctx* ctx);

/* Reads back the decoder config (as set by vxb_set_config / vxb_load_gguf):
 * latent and decoder widths and up to max_rates upsampling rates; *n_rates
 * receives the number of rates.  The reference reads the same fields from
 * AudioVAEConfig (include/voxcpm/config.h:34-133). */
VXB_API int vxb_get_config(const vxb_ctx* ctx, int* latent_dim, int* decoder_dim, int* rates, int max_rates,
                           int* n_rates);

/* One decode of the planned shape: z [batch][latent_dim][T] (t fastest, each
 * one the reference's ne=[T,latent_dim]) -> out [batch][hop*T], both HOST
 * pointers; includes the host->device and device->host copies and waits for
 * completion (bounded, VXB_ERR_TIMEOUT after 60 s).  Replaces
 * tensor_set(latent) + VoxCPMBackend::compute + tensor_get(audio)
 * (src/backend.cpp:293-339, vae_decode_mock.cpp:1186-1202). */
VXB_API int vxb_decode(vxb_ctx* ctx, const float* z_host, float* out_host);

/* Same with DEVICE pointers, enqueued on `stream` (NULL = the context's
 * stream) without waiting.  Check completion with vxb_sync. */
VXB_API int vxb_decode_device(vxb_ctx* ctx, const float* z_dev, float* out_dev, void* stream);

/* Waits for the context's stream (and `stream` if given) up to timeout_ms;
 * VXB_ERR_TIMEOUT if it has not finished, VXB_ERR_DEVICE_STATUS if a kernel
 * reported a failed bounded wait. */
VXB_API int vxb_sync(vxb_ctx* ctx, int timeout_ms);

/* Failure-detection probe: launches one kernel whose thread waits on an
 * mbarrier that nothing arrives on, through the bounded wait every decode
 * kernel uses, with the limit shortened to limit_us microseconds
 * (1..2000000).  The wait gives up, the kernel records a failed wait in the
 * context's device status word and returns -- no fault, no trap -- so the
 * next vxb_sync returns VXB_ERR_DEVICE_STATUS and the context stays usable
 * (the next decode clears the status word).  Enqueued on `stream` (NULL =
 * the context's stream).  No counterpart in the reference, whose CPU graph
 * has no device waits; its error convention is voxcpm::Error / ErrorCode
 * (include/voxcpm/common.h:42-88). */
VXB_API int vxb_debug_wait_probe(vxb_ctx* ctx, int limit_us, void* stream);

/* Copies the fp32 activation after plan stage `stage` (2+4b: transposed conv
 * of block b; 3+4b, 4+4b: residual units 0 and 1 of block b) of the last
 * decode to host memory [batch*frames][channels]; n = capacity in floats.
 * Other stages are fused away and return VXB_ERR_INVALID_ARGUMENT. */
VXB_API int vxb_debug_stage(vxb_ctx* ctx, int stage, float* host_out, size_t n);

/* Number of kernel launches in the current plan (one decode). */
VXB_API int vxb_plan_num_ops(const vxb_ctx* ctx);

/* Name, kernel (template instance as a profiler shows it) and algorithmic
 * work of plan op `idx`: flops = 2*M*K*N for the convs (elementwise work
 * counted roughly), bytes = minimal HBM traffic (weights once, each
 * activation read/written once). */
VXB_API int vxb_plan_op_info(const vxb_ctx* ctx, int idx, char* name, int name_cap, char* kernel, int kernel_cap,
                             double* flops, double* bytes);

/* Runs the plan's launch list `reps` times on the last decoded latent with a
 * CUDA event between consecutive launches and writes each op's mean device
 * time (ms) to ms_out[vxb_plan_num_ops]; if flush is given, flush_bytes of it
 * are overwritten before every rep to evict L2. */
VXB_API int vxb_time_ops(vxb_ctx* ctx, int reps, void* flush, size_t flush_bytes, float* ms_out);

/* Allocation-free decode, for callers that must not allocate device memory
 * once they are running: a real-time audio thread (cudaMalloc can stall and
 * synchronise the device) or a host whose device memory is all owned by
 * another allocator.  It runs the same kernels as vxb_decode_device, with
 * z_dev [batch][latent_dim][T] and out_dev [batch][hop*T] in device memory,
 * but keeps every intermediate activation in one fixed array compiled into
 * libvxb (5.63 MiB, present on every GPU that loads the library until the
 * process exits) instead of a plan arena, and calls no allocating routine.
 * Limit: batch*T <= 8 latent frames for the VoxCPM decoder (1536 channels,
 * rates 8,8,5,2); larger shapes return VXB_ERR_INVALID_ARGUMENT.  The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress),
 * so make that first call before any stream capture.  All calls share the
 * array: calls whose work overlaps on the GPU (other streams, other contexts
 * on the same device) race and corrupt each other; serialise them.  Enqueued
 * on `stream` (NULL = the context's stream); completion via vxb_sync or the
 * stream.  This entry point has no counterpart in the reference, which
 * always allocates its compute arena (src/backend.cpp:241-287). */
VXB_API int vxb_decode_static(vxb_ctx* ctx, const float* z_dev, float* out_dev, int batch, int T, void* stream);

/* ---- opt-in stateful streaming ---- */

/* One latent stream decoded n frames per push, carrying every causal layer's
 * left context from push to push (6 latent frames for model.0, 1 input row
 * per transposed conv, 6*d rows per residual unit's dilated conv, 6 rows for
 * the final conv) instead of re-decoding earlier frames: the pushes of a
 * stream emit exactly the continuous decode of all its frames so far.  This
 * is NOT the reference's streaming behaviour, which decodes every window of
 * vae_decode_mock.cpp alone with zero left context (vae_decode_mock.cpp:13-15,
 * :1337-1347); it has no counterpart there.  A stream object owns its
 * windows (two sets of a few MB for n = 6) and two CUDA graphs; it shares the
 * context's weights, device, stream and status word, so pushes of several
 * streams of one context must not overlap.  Requires vxb_prepare. */
typedef struct vxb_stream vxb_stream;

VXB_API int vxb_stream_open(vxb_ctx* ctx, int n_frames, vxb_stream** out);

/* Decodes the next n_frames of the stream: z [latent_dim][n_frames] (t
 * fastest) -> out [hop * n_frames], HOST pointers, blocking (60 s bound). */
VXB_API int vxb_stream_push(vxb_stream* s, const float* z_host, float* out_host);

/* Same with DEVICE pointers, enqueued on `stream` (NULL = the context's
 * stream) without waiting; completion via vxb_sync on the context. */
VXB_API int vxb_stream_push_device(vxb_stream* s, const float* z_dev, float* out_dev, void* stream);

/* Forgets the stream's history: the next push starts a new stream. */
VXB_API int vxb_stream_reset(vxb_stream* s);

VXB_API int vxb_stream_close(vxb_stream* s);

/* ---- encoder: waveform -> latent ---- */

/* Sets the encoder config for callers that upload tensors themselves
 * (vxb_load_gguf reads it from voxcpm_audio_vae_config_encoder_dim / _rates):
 * head width and the downsampling rates, in the roles of AudioVAEConfig's
 * encoder_dim / encoder_rates (include/voxcpm/config.h:34-133). */
VXB_API int vxb_set_encoder_config(vxb_ctx* ctx, int encoder_dim, const int* rates, int n_rates);

/* Reads back the encoder config (vxb_set_encoder_config / vxb_load_gguf):
 * *encoder_dim and up to max_rates downsampling rates, *n_rates = their
 * count (0 and 0 without an encoder config). */
VXB_API int vxb_get_encoder_config(const vxb_ctx* ctx, int* encoder_dim, int* rates, int max_rates, int* n_rates);

/* Waveform samples per latent frame: the product of the encoder rates
 * (AudioVAEConfig::hop_length); 0 without an encoder config. */
VXB_API int vxb_encoder_hop(const vxb_ctx* ctx);

/* Binds the encoder weights (audio_vae.encoder.*, the names
 * load_encoder_weights reads, src/audio-vae.cpp:331-363; F16 conv weights
 * [K, Cin, Cout] or Q4_0 folded [K*Cin, Cout], :64-103) on its first call
 * after vxb_prepare, then allocates the activation arena for `batch`
 * waveforms of T * vxb_encoder_hop samples each.  Replaces the graph build +
 * gallocr reserve of AudioVAE::encode (src/audio-vae.cpp:652-664) for that
 * shape.  VXB_ERR_INVALID_FORMAT if the model's encoder tensors are
 * placeholders or an encoder width is not a multiple of 32. */
VXB_API int vxb_build_encode_plan(vxb_ctx* ctx, int batch, int T);

/* One encode of the planned shape: audio [batch][T*hop] (16 kHz samples;
 * pad a shorter waveform with zeros to the hop multiple, as the reference's
 * AudioVAE::preprocess does, src/audio-vae.cpp:465-474) -> latent
 * [batch][latent_dim][T] (t fastest: each one the reference's ne=[T, latent],
 * the input layout of vxb_decode), both HOST pointers; copies in, runs,
 * copies out and waits (bounded, VXB_ERR_TIMEOUT after 60 s).  Replaces
 * AudioVAE::encode + VoxCPMBackend::compute + tensor_get
 * (src/audio-vae.cpp:640-664, src/backend.cpp:293-339). */
VXB_API int vxb_encode(vxb_ctx* ctx, const float* audio_host, float* latent_host);

/* Same with DEVICE pointers, enqueued on `stream` (NULL = the context's
 * stream) without waiting; completion via vxb_sync. */
VXB_API int vxb_encode_device(vxb_ctx* ctx, const float* audio_dev, float* latent_dev, void* stream);

/* The encode plan's launches, as vxb_plan_num_ops / vxb_plan_op_info /
 * vxb_time_ops for the decode plan. */
VXB_API int vxb_encode_num_ops(const vxb_ctx* ctx);
VXB_API int vxb_encode_op_info(const vxb_ctx* ctx, int idx, char* name, int name_cap, char* kernel, int kernel_cap,
                               double* flops, double* bytes);
VXB_API int vxb_encode_time_ops(vxb_ctx* ctx, int reps, void* flush, size_t flush_bytes, float* ms_out);

/* ---- single-kernel entry points (device pointers, enqueued on `stream`) ---- */

/* Q4_0 blocks -> fp32 ((q - 8) * d), bit-exact with ggml's
 * dequantize_row_q4_0 (ggml-quants.c:459-477). n = element count (multiple of 32). */
VXB_API int vxb_q4_0_dequant(const void* blocks, int64_t n, float* out, void* stream);

/* y[n][c] = x + sin(alpha*x)^2 / (alpha + 1e-9) over fp32 [N][C]
 * (snake_fused_l2_custom, src/audio-vae.cpp:1443-1479). */
VXB_API int vxb_snake(const float* x, const float* alpha, int C, int64_t N, float* y, void* stream);

/* Pointwise conv as ggml mul_mat + bias (+ residual) (+ Snake) on the tensor
 * cores: y[n][m] = sum_k W[m][k] x[n][k] + bias[m] (+ res[n][m]), then
 * optionally Snake(alpha) and fp16 output.  W is the GGUF [K, M] weight (F16
 * or Q4_0 bytes), x fp16 [N][K].  Replaces pointwise_l2 (src/audio-vae.cpp:1421-1435). */
VXB_API int vxb_pointwise(const void* w, int w_type, int K, int M, const void* x_f16, int64_t N, const float* bias,
                  const float* res, const float* snake_alpha, int out_f16, void* y, void* stream);

/* One residual unit on device buffers (reference residual_unit_forward_l2,
 * src/audio-vae.cpp:1481-1518): y = x + pw(snake2(dw_d(snake1(x)))) + pb,
 * then, when out_alpha is given, the next layer's Snake with that alpha
 * (fp16 output if out_f16, else fp32).  x and y are [batch][T][C], channels
 * fastest; w is the unit's pointwise weight as GGUF bytes (F16 [C][C] or
 * Q4_0 rows of C/32 blocks); dw the depthwise taps [C][7] fp32; a1, a2, db,
 * pb, out_alpha fp32 [C]; 1 <= d <= 9.  Runs the fused residual-unit kernel
 * for C <= 128 (C % 32 == 0), the prologue + pointwise-only kernel for
 * C <= 192 when the batch has a tile of 128 tokens per SM, else the prologue
 * + pointwise GEMM.  Enqueued on `stream`; temporaries are stream-ordered. */
VXB_API int vxb_residual_unit(const void* w, int w_type, int C, int d, const float* x, int batch, int T,
                              const float* a1, const float* dw, const float* db, const float* a2, const float* pb,
                              const float* out_alpha, int out_f16, void* y, void* stream);

/* Causal transposed conv (kernel 2s, stride s, cropped to T*s) as one
 * implicit GEMM with a col2im epilogue: x fp16 [B*T][Cin] -> y fp32
 * [B*T*s][Cout]; W is the folded GGUF [2s*Cout, Cin] weight (F16 or Q4_0).
 * Replaces causal_transpose_conv1d_l2 / causal_transpose_conv1d
 * (src/audio-vae.cpp:1642-1673, :512-534). */
VXB_API int vxb_convt(const void* w, int w_type, int Cin, int Cout, int s, const void* x_f16, int B, int T,
              const float* bias, float* y, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VXB_H */
