// libvxb: the C ABI of include/vxb.h.  Weight store (unchanged F16 / Q4_0
// bytes in HBM), derived vectors, the fixed launch plan of one decode and its
// CUDA graph, and the single-kernel entry points.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <array>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "elementwise.cuh"
#include "encoder.cuh"
#include "gemm.cuh"
#include "resunit.cuh"
#include "convt_tm.cuh"
#include "gguf_reader.h"
#include "vxb.h"

using namespace vxb;

// ------------------------------------------------------------------ errors --

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

#define CUDA_TRY(expr)                                                                              \
    do {                                                                                            \
        cudaError_t e_ = (expr);                                                                    \
        if (e_ != cudaSuccess)                                                                      \
            return fail(e_ == cudaErrorMemoryAllocation ? VXB_ERR_OUT_OF_MEMORY : VXB_ERR_BACKEND, \
                        std::string(#expr) + ": " + cudaGetErrorString(e_));                       \
    } while (0)

// --------------------------------------------------------------- tensor maps --

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D fp16 tensor [outer][inner] (inner contiguous) with a {box_inner, box_outer}
// box and the 128-byte swizzle; out-of-range elements read as zero.
int make_tmap_f16(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                  uint32_t box_inner, uint32_t box_outer) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(VXB_ERR_BACKEND, "cuTensorMapEncodeTiled unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15))
        return fail(VXB_ERR_INVALID_ARGUMENT, "TMA operand needs 16-byte aligned base and row pitch");
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(VXB_ERR_BACKEND, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
    return VXB_OK;
}

// 2-D fp32 / fp16 tensor [outer][inner] without swizzle (epilogue tiles).
int make_tmap_plain(CUtensorMap* m, const void* base, bool f16, uint64_t inner, uint64_t outer, uint32_t box_inner,
                    uint32_t box_outer) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(VXB_ERR_BACKEND, "cuTensorMapEncodeTiled unavailable");
    const uint64_t row_bytes = inner * (f16 ? 2 : 4);
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15))
        return fail(VXB_ERR_INVALID_ARGUMENT, "epilogue tensor needs 16-byte aligned base and rows");
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                     const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(VXB_ERR_BACKEND, "cuTensorMapEncodeTiled (plain) failed: " + std::to_string(r));
    return VXB_OK;
}

// 2-D fp32 tensor [outer][inner] with the 128-byte swizzle (box rows of 128 B).
int make_tmap_f32_sw128(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                        uint32_t box_outer) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(VXB_ERR_BACKEND, "cuTensorMapEncodeTiled unavailable");
    const uint64_t row_bytes = inner * 4;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15) || box_inner * 4 != 128)
        return fail(VXB_ERR_INVALID_ARGUMENT, "swizzled fp32 tensor needs 16-byte aligned rows and 128-byte boxes");
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(VXB_ERR_BACKEND, "cuTensorMapEncodeTiled (f32 sw128) failed: " + std::to_string(r));
    return VXB_OK;
}

// 2-D byte tensor [rows][pitch] (no swizzle), for the raw Q4_0 blocks.
int make_tmap_u8(CUtensorMap* m, const void* base, uint64_t pitch, uint64_t rows, uint32_t box_inner,
                 uint32_t box_outer) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(VXB_ERR_BACKEND, "cuTensorMapEncodeTiled unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (pitch & 15))
        return fail(VXB_ERR_INVALID_ARGUMENT, "Q4_0 rows must be padded to 16 bytes for TMA");
    const cuuint64_t dims[2] = {pitch, rows};
    const cuuint64_t strides[1] = {pitch};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(VXB_ERR_BACKEND, "cuTensorMapEncodeTiled (u8) failed: " + std::to_string(r));
    return VXB_OK;
}

int num_sms(int dev) {
    static int cache[64] = {};
    if (dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

// A conv weight as a GEMM operand: fp16 bytes, or Q4_0 blocks split into
// their 16 nibble bytes (p: [rows][pitch bytes], block b at 16 * b, pitch
// >= 16 * blocks) and their fp16 scales transposed (s: [blocks][spitch
// bytes], spitch a multiple of 16) -- both 16-byte aligned for TMA, the
// values unchanged.
struct WView {
    const void* p = nullptr;
    int type = 0;
    int pitch = 0;
    const void* s = nullptr;
    int spitch = 0;
};

// Q4_0 rows [rows][nblk x 18 B] -> nibbles [rows][pitch B] (block bi at
// bi * 16, its values 8w..8w+7 in word w in the q4_slot order) + scales
// transposed [nblk][spitch / 2] fp16 (block bi of row r at bi * spitch + 2r),
// one thread per block (the nibbles and scales are moved, not re-quantised).
__global__ void q4_split_kernel(const uint8_t* __restrict__ src, int64_t rows, int nblk, uint8_t* __restrict__ q,
                                int pitch, uint8_t* __restrict__ sc, int spitch) {
    const int64_t total = rows * nblk;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / nblk;
        const int bi = static_cast<int>(i - r * nblk);
        const uint8_t* blk = src + i * 18;
        // value e of the block: low nibble of byte e (e < 16), high nibble of byte e - 16
        uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            const uint32_t v = e < 16 ? (blk[2 + e] & 15u) : (blk[2 + e - 16] >> 4);
            w[e >> 3] |= v << (4 * q4_slot(e & 7));
        }
        *reinterpret_cast<uint4*>(q + r * pitch + bi * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        sc[int64_t(bi) * spitch + r * 2] = blk[0];  // scales transposed: [block][row]
        sc[int64_t(bi) * spitch + r * 2 + 1] = blk[1];
    }
}

// Q4_0 rows -> fp16, (q - 8) * d rounded once (the value the GEMM's
// in-kernel dequantiser produces), same element order: the F16 layout of a
// tensor of the same shape.  One thread per block.
__global__ void q4_to_f16_kernel(const uint8_t* __restrict__ src, int64_t nblk, __half* __restrict__ out) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < nblk; i += int64_t(gridDim.x) * blockDim.x) {
        const uint8_t* blk = src + i * 18;
        const float d = __half2float(__ushort_as_half(static_cast<uint16_t>(blk[0] | (blk[1] << 8))));
        __half v[32];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            v[j] = __float2half_rn(static_cast<float>(static_cast<int>(blk[2 + j] & 15u) - 8) * d);
            v[j + 16] = __float2half_rn(static_cast<float>(static_cast<int>(blk[2 + j] >> 4) - 8) * d);
        }
        uint4* o = reinterpret_cast<uint4*>(out + i * 32);
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = reinterpret_cast<const uint4*>(v)[j];
    }
}

// Device buffers of a split Q4_0 weight.
struct SplitQ4 {
    void* q = nullptr;
    void* s = nullptr;
    int pitch = 0, spitch = 0;
};

// Splits a Q4_0 weight of `rows` rows of `inner` values (stream-ordered).
int split_q4(const void* w, int64_t inner, int64_t rows, cudaStream_t st, bool async_alloc, SplitQ4* out) {
    if (inner % 32) return fail(VXB_ERR_INVALID_ARGUMENT, "Q4_0 rows must hold whole blocks");
    const int nblk = static_cast<int>(inner / 32);
    // rows at least as wide as the GEMMs' widest TMA boxes (80 nibble bytes,
    // 16 scales); the padding is zero and lies past the matrix
    out->pitch = std::max(nblk * 16, kQ4MNNibBox);
    out->spitch = static_cast<int>(std::max<int64_t>((rows * 2 + 15) / 16 * 16, 256));  // bytes per block row
    const size_t qb = size_t(out->pitch) * rows, sb = size_t(out->spitch) * nblk;
    if (async_alloc) {
        CUDA_TRY(cudaMallocAsync(&out->q, qb, st));
        CUDA_TRY(cudaMallocAsync(&out->s, sb, st));
    } else {
        CUDA_TRY(cudaMalloc(&out->q, qb));
        CUDA_TRY(cudaMalloc(&out->s, sb));
    }
    CUDA_TRY(cudaMemsetAsync(out->s, 0, sb, st));
    if (out->pitch != nblk * 16) CUDA_TRY(cudaMemsetAsync(out->q, 0, qb, st));
    const int64_t total = rows * nblk;
    const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 16));
    q4_split_kernel<<<std::max(grid, 1), 256, 0, st>>>(static_cast<const uint8_t*>(w), rows, nblk,
                                                        static_cast<uint8_t*>(out->q), out->pitch,
                                                        static_cast<uint8_t*>(out->s), out->spitch);
    CUDA_TRY(cudaGetLastError());
    return VXB_OK;
}

// The fp16 copy of a Q4_0 weight of `nelem` values (synchronous allocation).
int q4_make_f16(const void* w, int64_t nelem, cudaStream_t st, void** out) {
    CUDA_TRY(cudaMalloc(out, size_t(nelem) * 2));
    const int64_t nblk = nelem / 32;
    const int grid = static_cast<int>(std::min<int64_t>((nblk + 255) / 256, 148 * 16));
    q4_to_f16_kernel<<<std::max(grid, 1), 256, 0, st>>>(static_cast<const uint8_t*>(w), nblk,
                                                         static_cast<__half*>(*out));
    CUDA_TRY(cudaGetLastError());
    return VXB_OK;
}

// --------------------------------------------------------------- launching --

int pick_bn(int64_t n) {
    if (n > 4096) return 256;
    if (n > 512) return 128;
    if (n > 48) return 64;
    if (n > 16) return 32;
    return 16;
}

// Halves a tile width (down to 32) while the layer's m_tiles x n_tiles tiles
// would leave SMs of the current device idle: on short sequences more,
// narrower tiles shorten every CTA's chain (fewer epilogue chunks per CTA).
// Token tiles advance by bn - overlap tokens.
int fill_bn(int bn, int m_tiles, int64_t N, int overlap) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int64_t sms = num_sms(dev);
    while (bn > 32 && int64_t(m_tiles) * ((N + bn - overlap - 1) / (bn - overlap)) < sms) bn /= 2;
    return bn;
}

// Launches a decode kernel with programmatic stream serialisation (the
// kernel calls grid_dep_sync before it touches activations), so its launch
// and setup overlap the previous kernel; captured into graphs as
// programmatic edges.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <int AK, int BN, int EPI, int RESKB = 0>
int launch_gemm_t(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tr, const CUtensorMap& to,
                  const CUtensorMap& ts,
                  const GemmArgs& a, cudaStream_t st, int grid_ctas = 0) {
    constexpr int smem = GemmCfg<BN, (AK >= kAQ4K), EPI, RESKB>::kSmemBytes;
    constexpr int threads = GemmCfg<BN, (AK >= kAQ4K), EPI, RESKB>::kThreads;
    static bool attr[64] = {};  // per device
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(VXB_ERR_BACKEND, "device index out of range");
    if (!attr[dev]) {
        CUDA_TRY(cudaFuncSetAttribute(gemm_kernel<AK, BN, EPI, RESKB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      smem));
        attr[dev] = true;
    }
    const int tiles = a.m_tiles * a.n_tiles;
    dim3 g(grid_ctas > 0 ? grid_ctas : std::max(1, std::min(tiles, num_sms(dev))));
    CUDA_TRY(launch_pdl(gemm_kernel<AK, BN, EPI, RESKB>, g, dim3(threads), smem, st, ta, tb, tr, to, ts, a));
    return VXB_OK;
}

template <int AK, int EPI>
int launch_gemm_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tr, const CUtensorMap& ts,
                   const CUtensorMap& to, const GemmArgs& a, cudaStream_t st) {
    switch (bn) {
        case 16:
            if constexpr (EPI == kEpiConvT) return launch_gemm_t<AK, 16, EPI>(ta, tb, tr, to, ts, a, st);
            return fail(VXB_ERR_INVALID_ARGUMENT, "pointwise tiles are at least 32 wide");
        case 32: return launch_gemm_t<AK, 32, EPI>(ta, tb, tr, to, ts, a, st);
        case 64: return launch_gemm_t<AK, 64, EPI>(ta, tb, tr, to, ts, a, st);
        case 128: return launch_gemm_t<AK, 128, EPI>(ta, tb, tr, to, ts, a, st);
        case 256:
            if constexpr (EPI == kEpiConvT) return launch_gemm_t<AK, 256, EPI>(ta, tb, tr, to, ts, a, st);
            return fail(VXB_ERR_INVALID_ARGUMENT, "pointwise tiles are at most 128 wide");
        default: return fail(VXB_ERR_INVALID_ARGUMENT, "bad BN");
    }
}

// A prepared GEMM launch (tensor maps and arguments fixed at plan time).
struct GemmOp;
std::string gemm_kernel_name(const GemmOp& op);

template <int SS, int CPT>
int launch_convt_tm_t(const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& ts, const CUtensorMap& ty,
                      const ConvTmArgs& a, int grid, cudaStream_t st) {
    constexpr int smem = ConvTmCfg<SS, CPT>::kSmemBytes;
    static bool attr[64] = {};  // per device
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(VXB_ERR_BACKEND, "device index out of range");
    if (!attr[dev]) {
        CUDA_TRY(cudaFuncSetAttribute(convt_tm_kernel<SS, CPT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr[dev] = true;
    }
    CUDA_TRY(launch_pdl(convt_tm_kernel<SS, CPT>, dim3(grid), dim3(kTmThreads), smem, st, tx, tw, ts, ty, a));
    return VXB_OK;
}

struct GemmOp {
    int akind = 0, epi = 0, bn = 16;
    int reskb = 0;    // > 0: resident-A kernel (Q4_0), grid = res_grid CTAs, each on one m tile
    int res_grid = 0;
    int tm_s = 0;     // > 0: transposed conv with the tokens as M (convt_tm_kernel<tm_s, tm.cpt>)
    ConvTmArgs tm{};
    dim3 grid;
    CUtensorMap ta{}, tb{}, tr{}, to{}, ts{};  // ts: Q4_0 scales (a copy of ta for fp16 weights)
    GemmArgs args{};
    int launch(cudaStream_t st) const {
        if (tm_s == 2 && tm.cpt == 32) return launch_convt_tm_t<2, 32>(tb, ta, ts, to, tm, res_grid, st);
        if (tm_s == 5 && tm.cpt == 16) return launch_convt_tm_t<5, 16>(tb, ta, ts, to, tm, res_grid, st);
        if (tm_s) return fail(VXB_ERR_INVALID_ARGUMENT, "unsupported tokens-as-M transposed conv");
        if (reskb == 6 && akind == kAQ4K && epi == kEpiPW && bn == 128)
            return args.out_f16 ? launch_gemm_t<kAQ4K, 128, kEpiPW, 6>(ta, tb, tr, to, ts, args, st, res_grid)
                                : launch_gemm_t<kAQ4K, 128, kEpiPW32, 6>(ta, tb, tr, to, ts, args, st, res_grid);
        if (reskb == 6 && akind == kAQ4MN && epi == kEpiConvT && bn == 256)
            return launch_gemm_t<kAQ4MN, 256, kEpiConvT, 6>(ta, tb, tr, to, ts, args, st, res_grid);
        if (reskb == 3 && akind == kAQ4MN && epi == kEpiConvT && bn == 256)
            return launch_gemm_t<kAQ4MN, 256, kEpiConvT, 3>(ta, tb, tr, to, ts, args, st, res_grid);
        if (reskb) return fail(VXB_ERR_INVALID_ARGUMENT, "unsupported resident-A GEMM");
        switch (akind * 2 + epi) {
            case kAF16K * 2 + kEpiPW: return launch_gemm_bn<kAF16K, kEpiPW>(bn, ta, tb, tr, ts, to, args, st);
            case kAQ4K * 2 + kEpiPW: return launch_gemm_bn<kAQ4K, kEpiPW>(bn, ta, tb, tr, ts, to, args, st);
            case kAF16MN * 2 + kEpiConvT: return launch_gemm_bn<kAF16MN, kEpiConvT>(bn, ta, tb, tr, ts, to, args, st);
            case kAQ4MN * 2 + kEpiConvT: return launch_gemm_bn<kAQ4MN, kEpiConvT>(bn, ta, tb, tr, ts, to, args, st);
            default: return fail(VXB_ERR_INVALID_ARGUMENT, "unsupported GEMM kind");
        }
    }
};

std::string gemm_kernel_name(const GemmOp& op) {
    if (op.tm_s) return "convt_tm_kernel<" + std::to_string(op.tm_s) + ", " + std::to_string(op.tm.cpt) + ">";
    // the resident-A pointwise kernel with fp32 output runs as kEpiPW32
    const int epi = (op.reskb && op.epi == kEpiPW && !op.args.out_f16) ? int(kEpiPW32) : op.epi;
    return "gemm_kernel<" + std::to_string(op.akind) + ", " + std::to_string(op.bn) + ", " + std::to_string(epi) +
           (op.reskb ? ", " + std::to_string(op.reskb) : std::string()) + ">";
}

// Resident A (Q4_0 weights): worth it when every CTA runs several n tiles
// of one m tile, so that its weight column is dequantised once instead of
// once per tile; the column (K) must fit RESKB k blocks of shared memory.
void choose_resident(GemmOp* op, int num_kb) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = num_sms(dev);
    const GemmArgs& a = op->args;
    const int per_m = sms / a.m_tiles;  // CTAs per m tile
    if (per_m < 1 || int64_t(a.n_tiles) < 2LL * per_m) return;
    int kb = 0;
    if (op->akind == kAQ4K && op->epi == kEpiPW && op->bn == 128 && num_kb <= 6) kb = 6;
    if (op->akind == kAQ4MN && op->epi == kEpiConvT && op->bn == 256 && num_kb <= 6) kb = num_kb <= 3 ? 3 : 6;
    if (!kb) return;
    op->reskb = kb;
    op->res_grid = per_m * a.m_tiles;
}

// Pointwise conv GEMM: W [M rows][K] (F16, or Q4_0 rows padded to w.pitch), x fp16 [N][K].
int setup_pointwise(GemmOp* op, WView w, int K, int M, const void* x16, int64_t N, const float* bias,
                    const float* res, const float* alpha, const float* inv, int out_f16, void* out, int* status) {
    if (K <= 0 || M <= 0 || N <= 0 || N > (int64_t(1) << 31) - 1)
        return fail(VXB_ERR_INVALID_ARGUMENT, "pointwise: bad extents");
    if (K % 8) return fail(VXB_ERR_INVALID_ARGUMENT, "pointwise: K must be a multiple of 8");
    op->epi = kEpiPW;
    op->bn = fill_bn(std::max(32, std::min(128, pick_bn(N))), (M + 127) / 128, N, 0);
    op->grid = dim3(1);
    int rc = make_tmap_f16(&op->tb, x16, K, N, uint64_t(K) * 2, 64, op->bn);
    if (rc) return rc;
    // epilogue tiles: [kEpiChunk tokens][128 channels] of the residual (fp32) and output
    if ((rc = make_tmap_plain(&op->to, out, out_f16 != 0, M, N, 128, kEpiChunk))) return rc;
    if (res) {
        if ((rc = make_tmap_plain(&op->tr, res, false, M, N, 128, kEpiChunk))) return rc;
    } else {
        op->tr = op->to;
    }
    GemmArgs& a = op->args;
    a = GemmArgs{};
    a.M = M;
    a.K = K;
    a.N = static_cast<int>(N);
    a.m_tiles = (M + 127) / 128;
    a.n_tiles = static_cast<int>((N + op->bn - 1) / op->bn);
    a.bias = bias;
    a.res = res;
    a.snake_alpha = alpha;
    a.snake_inv = inv;
    a.out = out;
    a.out_f16 = out_f16;
    a.status = status;
    if (w.type == VXB_TYPE_F16) {
        op->akind = kAF16K;
        rc = make_tmap_f16(&op->ta, w.p, K, M, uint64_t(K) * 2, 64, 128);
        op->ts = op->ta;
    } else if (w.type == VXB_TYPE_Q4_0) {
        if (K % 32) return fail(VXB_ERR_INVALID_ARGUMENT, "Q4_0 pointwise needs K % 32 == 0");
        op->akind = kAQ4K;
        choose_resident(op, (K + 63) / 64);
        // per k step: 2 blocks of nibbles (32 B) for 128 rows, and their scales (2 block rows of 128)
        rc = make_tmap_u8(&op->ta, w.p, w.pitch, M, kQ4KNibBox, 128);
        if (!rc) rc = make_tmap_plain(&op->ts, w.s, true, uint64_t(w.spitch) / 2, K / 32, 128, kQ4KScaleRows);
        return rc;
    } else {
        return fail(VXB_ERR_INVALID_ARGUMENT, "pointwise: weight type must be F16 or Q4_0");
    }
    return rc;
}

// Couts per transposed-conv tile: 2s*cpt rows <= 128 and a multiple of 8
// (so that every A tile starts on a 16-byte boundary).
int convt_cpt(int s) {
    for (int c = 128 / (2 * s); c > 0; --c)
        if ((2 * s * c) % 8 == 0 && c % 4 == 0) return c;
    return 0;
}

// Transposed conv GEMM: W folded [Cin rows][2s*Cout] (F16, or Q4_0 rows padded
// to w.pitch), x fp16 [B*T][Cin].
int setup_convt(GemmOp* op, WView w, int Cin, int Cout, int s, const void* x16, int B, int T, const float* bias,
                float* y, int* status, int skip = 0) {
    const int64_t N = int64_t(B) * T;
    if (skip < 0 || skip >= T) return fail(VXB_ERR_INVALID_ARGUMENT, "convt: bad skip");
    if (Cin <= 0 || Cout <= 0 || s <= 0 || s > 32 || N <= 0 || N * s > (int64_t(1) << 31) - 1)
        return fail(VXB_ERR_INVALID_ARGUMENT, "convt: bad extents");
    if (Cin % 8) return fail(VXB_ERR_INVALID_ARGUMENT, "convt: Cin must be a multiple of 8");
    if (Cout % 4) return fail(VXB_ERR_INVALID_ARGUMENT, "convt: Cout must be a multiple of 4");
    const int M = 2 * s * Cout;
    const int cpt = convt_cpt(s);
    if (cpt == 0) return fail(VXB_ERR_INVALID_ARGUMENT, "convt: stride too large");
    op->epi = kEpiConvT;
    if (w.type == VXB_TYPE_Q4_0 && skip == 0 && M % 32 == 0) {
        // Long stages of stride 2 and 5: the tokens-as-M kernel (its epilogue
        // needs no gather); every CTA keeps one j tile's dequantised weight
        // column (K <= 384) and walks at least two token tiles.
        const int tcpt = s == 2 ? 32 : s == 5 ? 16 : 0;
        int dev = 0;
        cudaGetDevice(&dev);
        const int sms = num_sms(dev);
        const int j_tiles = tcpt ? Cout / tcpt : 0;
        const int64_t n_tiles = (N + kTmTokens - 1) / kTmTokens;
        const int per_j = j_tiles ? sms / j_tiles : 0;
        // (stride 5 stores 32 bytes per output row: a 32-byte aligned output)
        const bool out_ok = s == 2 || (Cout % 8 == 0 && (reinterpret_cast<uintptr_t>(y) & 31) == 0);
        if (tcpt && out_ok && Cout % tcpt == 0 && Cin % 64 == 0 && Cin <= 64 * tm_max_kb(s) && per_j >= 1 &&
            n_tiles >= 2LL * per_j && n_tiles < (int64_t(1) << 30) / j_tiles) {
            op->tm_s = s;
            ConvTmArgs& t = op->tm;
            t = ConvTmArgs{};
            t.K = Cin;
            t.N = static_cast<int>(N);
            t.T = T;
            t.s = s;
            t.cout = Cout;
            t.cpt = tcpt;
            t.j_tiles = j_tiles;
            t.n_tiles = static_cast<int>(n_tiles);
            t.bias = bias;
            t.out = y;
            t.status = status;
            op->res_grid = per_j * j_tiles;
            op->bn = 2 * s * tcpt;
            int rc = make_tmap_f16(&op->tb, x16, Cin, N, uint64_t(Cin) * 2, 64, 32);
            if (!rc) rc = make_tmap_u8(&op->ta, w.p, w.pitch, Cin, kQ4MNNibBox, 64);
            if (!rc) rc = make_tmap_plain(&op->ts, w.s, true, uint64_t(w.spitch) / 2, M / 32, 64, kQ4MNScaleRows);
            // stride 2: one TMA store box of 31 tokens' output rows (32 couts, 128-byte
            // swizzle) per epilogue warp; stride 5 stores directly
            if (!rc && tcpt * 4 == 128) rc = make_tmap_f32_sw128(&op->to, y, Cout, uint64_t(N) * s, tcpt, 31 * s);
            if (tcpt * 4 != 128) op->to = op->tb;  // unused
            // GemmArgs filled for the plan's bookkeeping (op info), not read by the kernel
            op->args = GemmArgs{};
            op->args.M = M;
            op->args.K = Cin;
            op->args.N = static_cast<int>(N);
            op->args.s = s;
            op->args.cout = Cout;
            op->args.status = status;
            return rc;
        }
    }
    const int m_tiles = (Cout + cpt - 1) / cpt;
    if (w.type == VXB_TYPE_Q4_0 && m_tiles >= 32) {
        // Q4_0 weights are dequantised once per (m tile, n tile): with many m
        // tiles the SMs are filled by m alone, so the widest token tiles keep
        // the dequantisation per FLOP lowest (b0/b1 at batch 32: 4 -> 1 and
        // 13 -> 7 passes over the weights)
        op->bn = N + 1 > 128 ? 256 : pick_bn(N + 1);
    } else {
        op->bn = fill_bn(pick_bn(N + 1), m_tiles, N, 1);
    }
    op->grid = dim3(1);
    int rc = make_tmap_f16(&op->tb, x16, Cin, N, uint64_t(Cin) * 2, 64, op->bn);
    if (rc) return rc;
    op->tr = op->to = op->tb;  // unused by the transposed-conv epilogue
    GemmArgs& a = op->args;
    a = GemmArgs{};
    a.M = M;
    a.K = Cin;
    a.N = static_cast<int>(N);
    a.m_tiles = (Cout + cpt - 1) / cpt;
    a.n_tiles = static_cast<int>((N + op->bn - 2) / (op->bn - 1));
    a.bias = bias;
    a.out = y;
    a.s = s;
    a.cout = Cout;
    a.cpt = cpt;
    a.seq_len = T;
    a.skip = skip;
    a.v8 = cpt == 8 && Cout % 8 == 0 && (reinterpret_cast<uintptr_t>(y) & 31) == 0;
    a.status = status;
    if (w.type == VXB_TYPE_F16) {
        if ((uint64_t(M) * 2) % 16) return fail(VXB_ERR_INVALID_ARGUMENT, "convt: 2s*Cout must be a multiple of 8");
        op->akind = kAF16MN;
        rc = make_tmap_f16(&op->ta, w.p, M, Cin, uint64_t(M) * 2, 64, 64);
        op->ts = op->ta;
    } else if (w.type == VXB_TYPE_Q4_0) {
        if (M % 32) return fail(VXB_ERR_INVALID_ARGUMENT, "Q4_0 convt needs 2s*Cout % 32 == 0");
        op->akind = kAQ4MN;
        choose_resident(op, (Cin + 63) / 64);
        // per k step: up to 5 blocks of nibbles (80 B) for 64 rows, and their scales (5 block rows of 64)
        rc = make_tmap_u8(&op->ta, w.p, w.pitch, Cin, kQ4MNNibBox, 64);
        if (!rc) rc = make_tmap_plain(&op->ts, w.s, true, uint64_t(w.spitch) / 2, M / 32, 64, kQ4MNScaleRows);
        return rc;
    } else {
        return fail(VXB_ERR_INVALID_ARGUMENT, "convt: weight type must be F16 or Q4_0");
    }
    return rc;
}

// ------------------------------------------------- fused residual unit --

// fp32 activations [B][T][C] as a 3-D tensor (C fastest) for the fused
// residual unit: box {32 channels, rows, 1 sequence}; rows outside [0, T)
// read as zero and are not written.  swizzle: the 128-byte swizzle of the
// residual / output boxes (none for the producers' slices).
int make_tmap_x3d(CUtensorMap* m, const void* base, uint64_t C, uint64_t T, uint64_t B, uint32_t box_rows,
                  bool swizzle, bool f16 = false) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(VXB_ERR_BACKEND, "cuTensorMapEncodeTiled unavailable");
    const uint64_t es = f16 ? 2 : 4;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (C * es) % 16)
        return fail(VXB_ERR_INVALID_ARGUMENT, "residual-unit tensor needs 16-byte aligned base and rows");
    const cuuint64_t dims[3] = {C, T, B};
    const cuuint64_t strides[2] = {C * es, C * es * T};
    const cuuint32_t box[3] = {32, box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                     const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(VXB_ERR_BACKEND, "cuTensorMapEncodeTiled (x3d) failed: " + std::to_string(r));
    return VXB_OK;
}

template <int EPI, bool HG, int NE, int NH>
int launch_resunit_t(const CUtensorMap& tx, const CUtensorMap& tr, const CUtensorMap& ty, const CUtensorMap& th,
                     const ResUnitArgs& a, int grid, cudaStream_t st) {
    static bool attr[64] = {};  // per device
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(VXB_ERR_BACKEND, "device index out of range");
    if (!attr[dev]) {
        CUDA_TRY(cudaFuncSetAttribute(resunit_kernel<EPI, HG, NE, NH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kRuSmemLimit));
        attr[dev] = true;
    }
    const RuLayout L = ru_layout(a.C, HG, NH);
    if (L.ne != NE || ru_nh(a.C, HG, EPI) != NH) return fail(VXB_ERR_BACKEND, "residual unit: ring size mismatch");
    const size_t smem = static_cast<size_t>(L.total);
    CUDA_TRY(launch_pdl(resunit_kernel<EPI, HG, NE, NH>, dim3(grid), dim3(kRuThreads), smem, st, tx, tr, ty, th, a));
    return VXB_OK;
}

struct ResUnitOp {
    int epi = 0, grid = 1;
    bool hg = false;  // pointwise-only variant (H from the prologue kernel)
    CUtensorMap tx{}, tr{}, ty{}, th{};
    ResUnitArgs args{};
    int launch(cudaStream_t st) const {
        // rings (residual boxes, H buffers): the fused unit (3, 2); pointwise-only
        // (6, 2) for C <= 128, above that (6, 1) plain and (3, 2) with Snake
        const int nh = ru_nh(args.C, hg, epi);
        const int ne = ru_layout(args.C, hg, nh).ne;
        const int ring = !hg ? 0 : (ne == kRuMaxNE ? (nh == kRuNH ? 1 : 2) : 3);
        switch (epi * 4 + ring) {
            case kResPlain * 4: return launch_resunit_t<kResPlain, false, kRuNE, kRuNH>(tx, tr, ty, th, args, grid, st);
            case kResSnakeF16 * 4:
                return launch_resunit_t<kResSnakeF16, false, kRuNE, kRuNH>(tx, tr, ty, th, args, grid, st);
            case kResSnakeF32 * 4:
                return launch_resunit_t<kResSnakeF32, false, kRuNE, kRuNH>(tx, tr, ty, th, args, grid, st);
            case kResPlain * 4 + 1:
                return launch_resunit_t<kResPlain, true, kRuMaxNE, kRuNH>(tx, tr, ty, th, args, grid, st);
            case kResSnakeF16 * 4 + 1:
                return launch_resunit_t<kResSnakeF16, true, kRuMaxNE, kRuNH>(tx, tr, ty, th, args, grid, st);
            case kResSnakeF32 * 4 + 1:
                return launch_resunit_t<kResSnakeF32, true, kRuMaxNE, kRuNH>(tx, tr, ty, th, args, grid, st);
            case kResPlain * 4 + 2: return launch_resunit_t<kResPlain, true, kRuMaxNE, 1>(tx, tr, ty, th, args, grid, st);
            case kResSnakeF16 * 4 + 3:
                return launch_resunit_t<kResSnakeF16, true, kRuNE, kRuNH>(tx, tr, ty, th, args, grid, st);
            case kResSnakeF32 * 4 + 3:
                return launch_resunit_t<kResSnakeF32, true, kRuNE, kRuNH>(tx, tr, ty, th, args, grid, st);
            default: return fail(VXB_ERR_INVALID_ARGUMENT, "unsupported fused residual unit");
        }
    }
    std::string kernel_name() const {
        const int nh = ru_nh(args.C, hg, epi);
        return "resunit_kernel<" + std::to_string(epi) + ", " + (hg ? "1" : "0") + ", " +
               std::to_string(ru_layout(args.C, hg, nh).ne) + ", " + std::to_string(nh) + ">";  // as ncu names it
    }
};

// Whether a stage of C channels runs its residual units as one fused kernel
// (the pointwise weights of the unit fit shared memory).
bool resunit_fits(int C) { return C > 0 && C <= 128 && C % 32 == 0 && ru_layout(C).slots >= 2; }

// Whether a stage runs its residual units as one fused kernel: when the
// weights fit and the stage is short.  On long stages (at least two 128-token
// tiles per SM) the prologue kernel + the pointwise-only variant is faster
// on B200 (measured at 96 channels, batch 256 x 6 frames: 325 vs 350 us per
// unit), as the prologue's register windows keep more independent work in
// flight than the fused kernel's producer warps; short (streaming) stages
// keep the fused kernel, one launch instead of two.
bool resunit_fits(int C);
bool resunit_hg_fits(int C);
bool use_fused_unit(int C, int64_t B, int64_t T, int sms) {
    if (!resunit_fits(C)) return false;
    const int64_t tiles = B * ((T + kRuTT - 1) / kRuTT);
    return !(resunit_hg_fits(C) && tiles >= 2 * int64_t(sms));
}

// Whether the pointwise conv (+ bias + residual [-> Snake]) of a stage of C
// channels runs as the pointwise-only variant of that kernel (tokens as M,
// all C output channels in one tile: h is read once, no padded m-tiles).
bool resunit_hg_fits(int C) {
    return C > 0 && C <= 192 && C % 32 == 0 && ru_layout(C, true).total <= kRuSmemLimit;
}

// Fused residual unit over x [B*T][C] -> y; w = the unit's pointwise weight
// (GGUF bytes: F16 [C][C] or Q4_0 rows), dilation d <= 9.
// With h16 (the prologue's fp16 output [B*T][C]) the pointwise-only variant.
int setup_resunit(ResUnitOp* op, const void* w, int w_type, int C, int d, const float* x, void* y, int epi,
                  const float* a1, const float* i1, const float* dw, const float* db, const float* a2,
                  const float* i2, const float* pb, const float* sa, const float* si, int B, int T, int sms,
                  int* status, const void* h16 = nullptr) {
    op->hg = h16 != nullptr;
    if (!(op->hg ? resunit_hg_fits(C) : resunit_fits(C)) || d < 1 || d > 9 || B <= 0 || T <= 0)
        return fail(VXB_ERR_INVALID_ARGUMENT, "fused residual unit: bad extents");
    if (w_type != VXB_TYPE_F16 && w_type != VXB_TYPE_Q4_0)
        return fail(VXB_ERR_INVALID_ARGUMENT, "fused residual unit: weight type must be F16 or Q4_0");
    if (epi != kResPlain && (!sa || !si)) return fail(VXB_ERR_INVALID_ARGUMENT, "fused residual unit: no Snake");
    op->epi = epi;
    ResUnitArgs& a = op->args;
    a = ResUnitArgs{};
    a.x = x;
    a.y = y;
    a.a1 = a1;
    a.i1 = i1;
    a.dw = dw;
    a.db = db;
    a.a2 = a2;
    a.i2 = i2;
    a.w = static_cast<const uint8_t*>(w);
    a.w_q4 = w_type == VXB_TYPE_Q4_0;
    a.pb = pb;
    a.sa = sa;
    a.si = si;
    a.T = T;
    a.C = C;
    a.d = d;
    a.t_tiles = (T + kRuTT - 1) / kRuTT;
    const int64_t tiles = int64_t(B) * a.t_tiles;
    if (tiles > (int64_t(1) << 30)) return fail(VXB_ERR_INVALID_ARGUMENT, "fused residual unit: too many tiles");
    a.tiles = static_cast<int>(tiles);
    a.status = status;
    op->grid = static_cast<int>(std::min<int64_t>(tiles, sms));
    int rc = make_tmap_x3d(&op->tx, x, C, T, B, kRuTT + 6 * d, false);
    if (rc) return rc;
    if (op->hg) {
        if ((rc = make_tmap_f16(&op->th, h16, C, uint64_t(B) * T, uint64_t(C) * 2, 64, kRuTT))) return rc;
    } else {
        op->th = op->tx;  // unused
    }
    if ((rc = make_tmap_x3d(&op->tr, x, C, T, B, kRuTT, true))) return rc;
    // output: one box of 32 channels x 32 rows per epilogue warp
    if (epi == kResSnakeF16) return make_tmap_x3d(&op->ty, y, C, T, B, 32, false, true);
    return make_tmap_x3d(&op->ty, y, C, T, B, 32, true);
}

// Whether a prologue launch needs 64-bit index arithmetic: its thread count
// (rounded to whole blocks) or a sequence's rows x channels reach 2^31.
bool res_pre_wide(int C, int B, int T, int d, int t_off, int sms) {
    const long long threads = res_pre_threads(C, T, B, d, res_pre_run(C, T, B, d, sms));
    return (threads + 255) / 256 * 256 >= (1LL << 31) || static_cast<long long>(T + t_off) * C >= (1LL << 31);
}
std::string res_pre_kernel_name(int C, int B, int T, int d, int t_off, int sms) {  // as ncu names it
    return res_pre_wide(C, B, T, d, t_off, sms) ? "res_pre_kernel<true>" : "res_pre_kernel<false>";
}

// Residual-unit prologue over x [B][T][C] -> h fp16, dilation d.
int launch_res_pre(const float* x, const float* a1, const float* i1, const float* dw, const float* db, const float* a2,
                   const float* i2, __half* h, int C, int B, int T, int d, int sms, cudaStream_t s, int t_off = 0) {
    if (C % 2) return fail(VXB_ERR_INVALID_ARGUMENT, "prologue: C must be even");
    const int run = res_pre_run(C, T, B, d, sms);
    const long long threads = res_pre_threads(C, T, B, d, run);
    if (threads > (1LL << 40)) return fail(VXB_ERR_INVALID_ARGUMENT, "prologue: too many threads");
    const cudaError_t e = launch_pdl(res_pre_wide(C, B, T, d, t_off, sms) ? res_pre_kernel<true> : res_pre_kernel<false>,
                                     dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), 0, s, x, a1, i1,
                                     dw, db, a2, i2, h, C, T, B, d, run, t_off);
    return e == cudaSuccess ? VXB_OK : fail(VXB_ERR_BACKEND, std::string("prologue launch: ") + cudaGetErrorString(e));
}

// Final-conv tile: 128 time steps per block on long stages, 64 where that
// leaves fewer than two blocks per SM (short streaming steps).
int final_tile(int B, int T, int sms) {
    return int64_t(B) * ((T + 127) / 128) >= 2LL * sms ? 128 : 64;
}

int grid_1d(int64_t work, int threads) {
    const int64_t b = (work + threads - 1) / threads;
    return static_cast<int>(std::min<int64_t>(std::max<int64_t>(b, 1), 148 * 32));
}

// Converts an F32/F16 vector on the device to fp32 (and 1/(x+eps) if inv).
__global__ void vec_to_f32_kernel(const void* src, int type, int64_t n, float* dst, float* inv) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const float v = type == VXB_TYPE_F32 ? static_cast<const float*>(src)[i]
                                             : __half2float(static_cast<const __half*>(src)[i]);
        dst[i] = v;
        if (inv) inv[i] = 1.0f / (v + 1e-9f);
    }
}

}  // namespace

// ------------------------------------------------------------------ context --

struct DevTensor {
    std::string name;
    int type = 0;
    int n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    void* dev = nullptr;     // the GGUF bytes, unchanged
    size_t nbytes = 0;
    SplitQ4 split;           // Q4_0 conv weights: the same blocks as 16-byte nibble rows + fp16 scales (vxb_prepare)
    void* f16 = nullptr;     // Q4_0 conv weights, opt-in (vxb_set_q4_fp16_cache): the values rounded once to fp16
    int64_t nelem() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
    // The operand the plan's GEMMs read: fp16 values, or a Q4_0 weight's
    // blocks in their split form (16-byte aligned for TMA), dequantised to
    // fp16 in shared memory inside the GEMM mainloop (or, when the context
    // keeps fp16 copies of Q4_0 weights, that copy: the same operand values).
    WView gemm_view() const {
        if (type == VXB_TYPE_Q4_0 && f16) return WView{f16, VXB_TYPE_F16, 0, nullptr, 0};
        if (type == VXB_TYPE_Q4_0) return WView{split.q, VXB_TYPE_Q4_0, split.pitch, split.s, split.spitch};
        return WView{dev, VXB_TYPE_F16, 0, nullptr, 0};
    }
    // Weight bytes one pass over gemm_view() reads (4.5 bits per Q4_0 value).
    double gemm_bytes() const {
        return type == VXB_TYPE_Q4_0 && !f16 ? double(nelem()) / 32 * 18 : double(nelem()) * 2;
    }
    void free_split() {
        cudaFree(split.q);
        cudaFree(split.s);
        cudaFree(f16);
        split = SplitQ4{};
        f16 = nullptr;
    }
};

struct Vec {  // derived fp32 vector (+ inverse for Snake alphas)
    float* v = nullptr;
    float* inv = nullptr;
};

struct ResUnit {
    Vec a1, db, a2, pb;
    float* dw = nullptr;  // [C][7] fp32
    const DevTensor* pw = nullptr;
};

struct Block {
    int cin = 0, cout = 0, s = 0;
    Vec alpha, bias;
    const DevTensor* convt = nullptr;
    ResUnit ru[3];
};

struct EncBlock {
    int cin = 0, cout = 0, s = 0;  // residual units at cin channels, then a conv k 2s stride s to cout
    ResUnit ru[3];
    Vec alpha, bias;
    const DevTensor* conv = nullptr;  // [Cout][Cin][2s] in memory
    __half* wperm = nullptr;          // its fp16 copy reordered [Cout][2s][Cin] (the im2col column order)
};

struct OpInfo {
    std::string name;
    double flops = 0, bytes = 0;  // algorithmic work: 2*M*K*N, minimal HBM traffic
    std::string kernel;           // kernel (template instance) the op launches
};

// Device buffers of one decode: the caller's latent and waveform, and the
// activation arena (each buffer sized for the largest stage).
struct DecodeBufs {
    const float* z = nullptr;  // [B][L][T]
    float* out = nullptr;      // [B][hop*T]
    float* xa = nullptr;       // fp32 residual stream (ping)
    float* xb = nullptr;       // fp32 residual stream (pong)
    __half* h16 = nullptr;     // fp16 pointwise B operand (prologue output, head output)
    __half* s16 = nullptr;     // fp16 transposed-conv B operand (encoder: the im2col operand)
    __half* g16 = nullptr;     // encoder: fp16 Snake output of a block's last residual unit
    int* status = nullptr;     // device status word
};

struct Plan {
    int B = 0, T = 0;
    bool use_graph = false;
    float* z = nullptr;     // [B][L][T]
    float* out = nullptr;   // [B][hop*T]
    DecodeBufs bufs;
    size_t bytes = 0;
    std::vector<std::function<int(cudaStream_t)>> ops;
    std::vector<OpInfo> info;   // one per op
    std::vector<GemmOp> gemms;  // stable storage referenced by ops
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    struct StageRef {
        float* buf;
        size_t floats;
        size_t last_op;  // index of the op that writes it
    };
    std::map<int, StageRef> stage_buf;  // debug stages
};

struct vxb_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    int latent_dim = 64, decoder_dim = 1536;
    std::vector<int> rates{8, 8, 5, 2};
    bool config_set = false;
    std::map<std::string, DevTensor> tensors;
    bool prepared = false;
    std::vector<void*> derived_allocs;
    // bound decoder
    float* dw0 = nullptr;
    Vec b0, b1;
    const DevTensor* pw1 = nullptr;
    std::vector<Block> blocks;
    Vec final_alpha;
    float* final_w = nullptr;
    float final_bias = 0.f;
    std::unique_ptr<Plan> plan;
    // encoder: config (GGUF keys or vxb_set_encoder_config), weights bound at
    // the first vxb_build_encode_plan after vxb_prepare, its own plan
    int encoder_dim = 0;
    std::vector<int> enc_rates;
    bool enc_bound = false;
    float* enc_w0 = nullptr;  // head conv [E][7]
    Vec enc_b0, fc_b;
    std::vector<EncBlock> enc_blocks;
    const DevTensor* fc_mu = nullptr;
    __half* fc_perm = nullptr;  // fc_mu weight [latent][3][C]
    std::unique_ptr<Plan> enc_plan;
    int* status = nullptr;         // device status word
    int* status_host = nullptr;    // pinned mirror
    bool q4_fp16_cache = false;    // vxb_set_q4_fp16_cache: plan GEMMs read fp16 copies of Q4_0 weights
};

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

void free_plan(Plan* p) {
    if (!p) return;
    if (p->exec) cudaGraphExecDestroy(p->exec);
    if (p->graph) cudaGraphDestroy(p->graph);
    cudaFree(p->z);
    cudaFree(p->out);
    cudaFree(p->bufs.xa);
    cudaFree(p->bufs.xb);
    cudaFree(p->bufs.h16);
    cudaFree(p->bufs.s16);
    cudaFree(p->bufs.g16);
}

const DevTensor* get(vxb_ctx* c, const std::string& name) {
    auto it = c->tensors.find(name);
    return it == c->tensors.end() ? nullptr : &it->second;
}

}  // namespace

extern "C" {

const char* vxb_last_error(void) { return g_last_error.c_str(); }

int vxb_open(int device, vxb_ctx** out) {
    if (!out) return fail(VXB_ERR_INVALID_ARGUMENT, "null out");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return fail(VXB_ERR_BACKEND, "no CUDA device");
    if (device < 0 || device >= n) return fail(VXB_ERR_INVALID_ARGUMENT, "bad device index");
    cudaDeviceProp prop;
    CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return fail(VXB_ERR_BACKEND, "libvxb needs an sm_100 (B200) device");
    DeviceGuard g(device);
    auto c = std::make_unique<vxb_ctx>();
    c->device = device;
    CUDA_TRY(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    CUDA_TRY(cudaMalloc(&c->status, sizeof(int)));
    CUDA_TRY(cudaMemset(c->status, 0, sizeof(int)));
    CUDA_TRY(cudaMallocHost(&c->status_host, sizeof(int)));
    *c->status_host = 0;
    *out = c.release();
    return VXB_OK;
}

int vxb_close(vxb_ctx* c) {
    if (!c) return VXB_OK;
    DeviceGuard g(c->device);
    cudaStreamSynchronize(c->stream);
    if (c->plan) free_plan(c->plan.get());
    if (c->enc_plan) free_plan(c->enc_plan.get());
    for (auto& kv : c->tensors) {
        cudaFree(kv.second.dev);
        kv.second.free_split();
    }
    for (void* p : c->derived_allocs) cudaFree(p);
    cudaFree(c->status);
    cudaFreeHost(c->status_host);
    cudaStreamDestroy(c->stream);
    delete c;
    return VXB_OK;
}

int vxb_set_q4_fp16_cache(vxb_ctx* c, int enable) {
    if (!c) return fail(VXB_ERR_INVALID_ARGUMENT, "null ctx");
    if (c->q4_fp16_cache != (enable != 0)) {
        c->q4_fp16_cache = enable != 0;
        c->prepared = false;  // the next vxb_prepare lays the weights out again
    }
    return VXB_OK;
}

int vxb_set_config(vxb_ctx* c, int latent_dim, int decoder_dim, const int* rates, int n_rates) {
    if (!c || latent_dim <= 0 || decoder_dim <= 0 || !rates || n_rates <= 0 || n_rates > 8)
        return fail(VXB_ERR_INVALID_ARGUMENT, "bad decoder config");
    int ch = decoder_dim;
    for (int i = 0; i < n_rates; ++i) {
        if (rates[i] <= 0 || rates[i] > 32 || ch % 2) return fail(VXB_ERR_INVALID_ARGUMENT, "bad decoder rates");
        ch /= 2;
    }
    c->latent_dim = latent_dim;
    c->decoder_dim = decoder_dim;
    c->rates.assign(rates, rates + n_rates);
    c->config_set = true;
    c->prepared = false;
    return VXB_OK;
}

int vxb_upload_tensor(vxb_ctx* c, const char* name, int type, const int64_t* ne, int n_dims, const void* host,
                      size_t nbytes) {
    if (!c || !name || !ne || n_dims < 1 || n_dims > 4 || (!host && nbytes))
        return fail(VXB_ERR_INVALID_ARGUMENT, "bad tensor upload arguments");
    DevTensor t;
    t.name = name;
    t.type = type;
    t.n_dims = n_dims;
    for (int d = 0; d < n_dims; ++d) {
        if (ne[d] <= 0) return fail(VXB_ERR_INVALID_ARGUMENT, std::string("bad shape for ") + name);
        t.ne[d] = ne[d];
    }
    const size_t want = ggml_type_nbytes(type, t.nelem());
    if (want == 0 || want != nbytes)
        return fail(VXB_ERR_INVALID_FORMAT, std::string("type/size mismatch for ") + name);
    DeviceGuard g(c->device);
    t.nbytes = nbytes;
    CUDA_TRY(cudaMalloc(&t.dev, nbytes));
    CUDA_TRY(cudaMemcpy(t.dev, host, nbytes, cudaMemcpyHostToDevice));
    auto it = c->tensors.find(t.name);
    if (it != c->tensors.end()) {
        cudaFree(it->second.dev);
        it->second.free_split();
    }
    c->tensors[t.name] = t;
    c->prepared = false;
    return VXB_OK;
}

int vxb_load_gguf(vxb_ctx* c, const char* path) {
    if (!c || !path) return fail(VXB_ERR_INVALID_ARGUMENT, "null argument");
    GgufFile f;
    std::string err;
    if (!f.open(path, &err)) {
        FILE* probe = std::fopen(path, "rb");
        if (!probe) return fail(VXB_ERR_FILE_NOT_FOUND, err);
        std::fclose(probe);
        return fail(VXB_ERR_INVALID_FORMAT, err);
    }
    auto u32 = [&](const char* k, int* v) {
        const GgufValue* x = f.kv(k);
        if (!x || (x->type != 4 && x->type != 5)) return false;  // u32 / i32
        *v = static_cast<int>(x->i);
        return true;
    };
    int latent = 0, dec = 0;
    const GgufValue* r = f.kv("voxcpm_audio_vae_config_decoder_rates");
    if (!u32("voxcpm_audio_vae_config_latent_dim", &latent) || !u32("voxcpm_audio_vae_config_decoder_dim", &dec) ||
        !r || r->arr_i.empty())
        return fail(VXB_ERR_INVALID_FORMAT, "GGUF lacks the required voxcpm_audio_vae_config_* keys");
    std::vector<int> rates(r->arr_i.begin(), r->arr_i.end());
    int rc = vxb_set_config(c, latent, dec, rates.data(), static_cast<int>(rates.size()));
    if (rc) return rc;
    // encoder config: optional (a decoder-only caller never needs it)
    int enc = 0;
    const GgufValue* er = f.kv("voxcpm_audio_vae_config_encoder_rates");
    if (u32("voxcpm_audio_vae_config_encoder_dim", &enc) && er && !er->arr_i.empty()) {
        std::vector<int> erates(er->arr_i.begin(), er->arr_i.end());
        if ((rc = vxb_set_encoder_config(c, enc, erates.data(), static_cast<int>(erates.size())))) return rc;
    }
    std::vector<uint8_t> buf;
    for (const auto& t : f.tensors) {
        if (t.nbytes == 0) continue;  // types this path never reads (encoder-only extras)
        buf.resize(t.nbytes);
        if (!f.read_tensor(t, buf.data(), &err)) return fail(VXB_ERR_INVALID_FORMAT, err);
        rc = vxb_upload_tensor(c, t.name.c_str(), t.type, t.ne, t.n_dims, buf.data(), t.nbytes);
        if (rc) return rc;
    }
    return VXB_OK;
}

int vxb_hop(const vxb_ctx* c) {
    if (!c) return 0;
    int h = 1;
    for (int r : c->rates) h *= r;
    return h;
}

int vxb_set_encoder_config(vxb_ctx* c, int encoder_dim, const int* rates, int n_rates) {
    if (!c || encoder_dim <= 0 || !rates || n_rates <= 0 || n_rates > 8)
        return fail(VXB_ERR_INVALID_ARGUMENT, "bad encoder config");
    for (int i = 0; i < n_rates; ++i)
        if (rates[i] <= 0 || rates[i] > 32) return fail(VXB_ERR_INVALID_ARGUMENT, "bad encoder rates");
    c->encoder_dim = encoder_dim;
    c->enc_rates.assign(rates, rates + n_rates);
    c->enc_bound = false;
    return VXB_OK;
}

int vxb_get_encoder_config(const vxb_ctx* c, int* encoder_dim, int* rates, int max_rates, int* n_rates) {
    if (!c || !encoder_dim || !n_rates || max_rates < 0 || (max_rates > 0 && !rates))
        return fail(VXB_ERR_INVALID_ARGUMENT, "vxb_get_encoder_config: null argument");
    *encoder_dim = c->encoder_dim;
    *n_rates = static_cast<int>(c->enc_rates.size());
    for (int i = 0; i < max_rates && i < *n_rates; ++i) rates[i] = c->enc_rates[i];
    return VXB_OK;
}

int vxb_encoder_hop(const vxb_ctx* c) {
    if (!c || c->enc_rates.empty()) return 0;
    int h = 1;
    for (int r : c->enc_rates) h *= r;
    return h;
}

int vxb_get_config(const vxb_ctx* c, int* latent_dim, int* decoder_dim, int* rates, int max_rates, int* n_rates) {
    if (!c || !latent_dim || !decoder_dim || !n_rates || max_rates < 0 || (max_rates > 0 && !rates))
        return fail(VXB_ERR_INVALID_ARGUMENT, "vxb_get_config: null argument");
    *latent_dim = c->latent_dim;
    *decoder_dim = c->decoder_dim;
    *n_rates = static_cast<int>(c->rates.size());
    for (int i = 0; i < max_rates && i < *n_rates; ++i) rates[i] = c->rates[i];
    return VXB_OK;
}

}  // extern "C"

namespace {

// Derived fp32 vector of tensor `name` with `n` elements.
int derive_vec(vxb_ctx* c, const std::string& name, int64_t n, bool with_inv, Vec* out) {
    const DevTensor* t = get(c, name);
    if (!t) return fail(VXB_ERR_MISSING_TENSOR, "missing tensor " + name);
    if ((t->type != VXB_TYPE_F32 && t->type != VXB_TYPE_F16) || t->nelem() != n)
        return fail(VXB_ERR_INVALID_FORMAT, "unexpected type/shape for " + name);
    CUDA_TRY(cudaMalloc(&out->v, n * sizeof(float)));
    c->derived_allocs.push_back(out->v);
    if (with_inv) {
        CUDA_TRY(cudaMalloc(&out->inv, n * sizeof(float)));
        c->derived_allocs.push_back(out->inv);
    }
    vec_to_f32_kernel<<<grid_1d(n, 256), 256, 0, c->stream>>>(t->dev, t->type, n, out->v, out->inv);
    CUDA_TRY(cudaGetLastError());
    return VXB_OK;
}

// Depthwise taps: GGUF [7, 1, C] (or [7, C, 1] for the final conv) is [c][k] in memory.
int derive_taps(vxb_ctx* c, const std::string& name, int C, float** out) {
    Vec v;
    const DevTensor* t = get(c, name);
    if (!t) return fail(VXB_ERR_MISSING_TENSOR, "missing tensor " + name);
    if (t->ne[0] != 7 || t->nelem() != int64_t(7) * C)
        return fail(VXB_ERR_INVALID_FORMAT, "unexpected shape for " + name);
    int rc = derive_vec(c, name, int64_t(7) * C, false, &v);
    *out = v.v;
    return rc;
}

// Binds a conv weight used as a GEMM operand ([outer rows][inner]); for Q4_0
// it also lays the same blocks out in their split form (nibble rows and
// scale rows, each 16-byte aligned) for the GEMMs' TMA loads.
int check_matrix(vxb_ctx* c, const std::string& name, int64_t inner, int64_t outer, const DevTensor** out) {
    auto it = c->tensors.find(name);
    if (it == c->tensors.end()) return fail(VXB_ERR_MISSING_TENSOR, "missing tensor " + name);
    DevTensor* t = &it->second;
    if (t->type != VXB_TYPE_F16 && t->type != VXB_TYPE_Q4_0)
        return fail(VXB_ERR_INVALID_FORMAT, name + ": conv weights must be F16 or Q4_0");
    if (t->nelem() != inner * outer) return fail(VXB_ERR_INVALID_FORMAT, "unexpected shape for " + name);
    if (t->type == VXB_TYPE_Q4_0) {
        if (inner % 32) return fail(VXB_ERR_INVALID_FORMAT, name + ": Q4_0 rows must hold whole blocks");
        t->free_split();
        if (c->q4_fp16_cache) {
            if (int rc = q4_make_f16(t->dev, t->nelem(), c->stream, &t->f16)) return rc;
        } else if (int rc = split_q4(t->dev, inner, outer, c->stream, false, &t->split)) {
            return rc;
        }
    }
    *out = t;
    return VXB_OK;
}

}  // namespace

extern "C" int vxb_prepare(vxb_ctx* c) {
    if (!c) return fail(VXB_ERR_INVALID_ARGUMENT, "null ctx");
    if (c->prepared) return VXB_OK;
    DeviceGuard g(c->device);
    for (void* p : c->derived_allocs) cudaFree(p);
    c->derived_allocs.clear();
    c->blocks.clear();
    // the encoder's derived weights went with the allocations above
    c->enc_bound = false;
    c->enc_blocks.clear();
    if (c->enc_plan) {
        free_plan(c->enc_plan.get());
        c->enc_plan.reset();
    }
    // The reference refuses a store whose encoder tensors are absent
    // (load_encoder_weights, src/audio-vae.cpp:331-363); the decoder never
    // reads them, so only their presence is checked.
    static const char* kEnc[] = {"audio_vae.encoder.block.0.weight", "audio_vae.encoder.block.0.bias",
                                 "audio_vae.encoder.fc_mu.weight", "audio_vae.encoder.fc_mu.bias"};
    for (const char* n : kEnc)
        if (!get(c, n)) return fail(VXB_ERR_MISSING_TENSOR, std::string("missing tensor ") + n);
    // Sample-rate conditioning (audio_vae.decoder.sr_cond_model.<i>.*, optional
    // in the reference, src/audio-vae.cpp:389-396) is not implemented: a model
    // that carries it is refused rather than decoded without it.
    for (const auto& kv : c->tensors)
        if (kv.first.rfind("audio_vae.decoder.sr_cond_model.", 0) == 0)
            return fail(VXB_ERR_INVALID_FORMAT, "sample-rate conditioning tensors are not supported: " + kv.first);
    const std::string p = "audio_vae.decoder.model.";
    const int L = c->latent_dim, D = c->decoder_dim;
    int rc;
    if ((rc = derive_taps(c, p + "0.weight", L, &c->dw0))) return rc;
    if ((rc = derive_vec(c, p + "0.bias", L, false, &c->b0))) return rc;
    if ((rc = check_matrix(c, p + "1.weight", L, D, &c->pw1))) return rc;
    if (!(c->pw1->ne[0] == L || (c->pw1->ne[0] == 1 && c->pw1->ne[1] == L)))
        return fail(VXB_ERR_INVALID_FORMAT, "model.1.weight must be [latent, decoder_dim] or [1, latent, decoder_dim]");
    if ((rc = derive_vec(c, p + "1.bias", D, false, &c->b1))) return rc;
    int C = D;
    for (size_t bi = 0; bi < c->rates.size(); ++bi) {
        Block b;
        b.cin = C;
        b.cout = C / 2;
        b.s = c->rates[bi];
        const std::string bp = p + std::to_string(bi + 2) + ".block.";
        if ((rc = derive_vec(c, bp + "0.alpha", C, true, &b.alpha))) return rc;
        if ((rc = check_matrix(c, bp + "1.weight", int64_t(2) * b.s * b.cout, C, &b.convt))) return rc;
        if (b.convt->ne[0] != (b.convt->n_dims == 3 ? 2 * b.s : 2 * b.s * b.cout))
            return fail(VXB_ERR_INVALID_FORMAT, bp + "1.weight: expected [2s*Cout, Cin] or [2s, Cout, Cin]");
        if ((rc = derive_vec(c, bp + "1.bias", b.cout, false, &b.bias))) return rc;
        for (int r = 0; r < 3; ++r) {
            const std::string rp = bp + std::to_string(r + 2) + ".block.";
            ResUnit& u = b.ru[r];
            if ((rc = derive_vec(c, rp + "0.alpha", b.cout, true, &u.a1))) return rc;
            if ((rc = derive_taps(c, rp + "1.weight", b.cout, &u.dw))) return rc;
            if ((rc = derive_vec(c, rp + "1.bias", b.cout, false, &u.db))) return rc;
            if ((rc = derive_vec(c, rp + "2.alpha", b.cout, true, &u.a2))) return rc;
            if ((rc = check_matrix(c, rp + "3.weight", b.cout, b.cout, &u.pw))) return rc;
            if ((rc = derive_vec(c, rp + "3.bias", b.cout, false, &u.pb))) return rc;
        }
        c->blocks.push_back(b);
        C /= 2;
    }
    // channel counts: 16-byte vectors in the elementwise kernels, TMA rows in the GEMMs
    if (C % 8 || C > 128 || L % 8)
        return fail(VXB_ERR_INVALID_FORMAT, "decoder channels must be multiples of 8 and the last stage <= 128");
    const int nb = static_cast<int>(c->rates.size());
    if ((rc = derive_vec(c, p + std::to_string(nb + 2) + ".alpha", C, true, &c->final_alpha))) return rc;
    if ((rc = derive_taps(c, p + std::to_string(nb + 3) + ".weight", C, &c->final_w))) return rc;
    const DevTensor* fb = get(c, p + std::to_string(nb + 3) + ".bias");
    if (!fb || fb->nelem() != 1) return fail(VXB_ERR_MISSING_TENSOR, "missing final conv bias");
    Vec fbv;
    if ((rc = derive_vec(c, fb->name, 1, false, &fbv))) return rc;
    CUDA_TRY(cudaMemcpyAsync(&c->final_bias, fbv.v, sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    c->prepared = true;
    return VXB_OK;
}

namespace {

// Largest activation of any stage (floats) and largest transposed-conv input.
void arena_sizes(const vxb_ctx* c, int B, int T, int64_t* max_x, int64_t* max_s) {
    *max_x = *max_s = int64_t(B) * T * c->decoder_dim;
    int64_t n = int64_t(B) * T;
    for (const Block& b : c->blocks) {
        *max_s = std::max(*max_s, n * b.cin);
        n *= b.s;
        *max_x = std::max(*max_x, n * b.cout);
    }
}

// Receives the launches of one decode in order.
struct OpSink {
    virtual ~OpSink() = default;
    virtual int gemm(const GemmOp& op, OpInfo info) = 0;
    virtual int kernel(std::function<int(cudaStream_t)> fn, OpInfo info) = 0;
    // the op emitted last writes debug stage `stage` into buf
    virtual void stage(int stage, float* buf, size_t floats) {}
};

// The launch sequence of one decode of B latents of T frames:
//   head dw -> model.1 pointwise (+ block 0 Snake, fp16)
//   per block: transposed conv -> 3 x (prologue: snake, dilated dw, snake ->
//              pointwise GEMM + bias + residual; the last unit also applies
//              the next block's Snake (fp16) or the final Snake (fp32))
//   final k7 conv + tanh.
int emit_decode(vxb_ctx* c, const DecodeBufs& d, int B, int T, OpSink& sink) {
    const int L = c->latent_dim, D = c->decoder_dim;
    const double n0 = double(B) * T;
    int rc;
    {
        const float *z = d.z, *w = c->dw0, *bb = c->b0.v;
        __half* o = d.h16;
        rc = sink.kernel(
            [=](cudaStream_t s) {
                const cudaError_t e =
                    launch_pdl(head_kernel, dim3(grid_1d(int64_t(B) * T * L, 256)), dim3(256), 0, s, z, w, bb, o, B, L, T, 0);
                return e == cudaSuccess ? VXB_OK : fail(VXB_ERR_BACKEND, "head launch");
            },
            {"head_dw", 14.0 * n0 * L, n0 * L * (4 + 2) + L * 8 * 4, "head_kernel"});
        if (rc) return rc;
    }
    {
        GemmOp op;
        const Block& b0 = c->blocks[0];
        if ((rc = setup_pointwise(&op, c->pw1->gemm_view(), L, D, d.h16, int64_t(B) * T, c->b1.v, nullptr,
                                  b0.alpha.v, b0.alpha.inv, 1, d.s16, d.status)))
            return rc;
        if ((rc = sink.gemm(op, {"pw_model1", 2.0 * D * L * n0, c->pw1->gemm_bytes() + n0 * L * 2 + n0 * D * 2,
                                 gemm_kernel_name(op)})))
            return rc;
    }
    int64_t n = int64_t(B) * T;
    int Tb = T;
    static const int kDil[3] = {1, 3, 9};
    const int sms = num_sms(c->device);
    for (size_t bi = 0; bi < c->blocks.size(); ++bi) {
        const Block& b = c->blocks[bi];
        const bool last_block = bi + 1 == c->blocks.size();
        {
            GemmOp op;
            if ((rc = setup_convt(&op, b.convt->gemm_view(), b.cin, b.cout, b.s, d.s16, B, Tb, b.bias.v, d.xa,
                                  d.status)))
                return rc;
            if ((rc = sink.gemm(op, {"convt_b" + std::to_string(bi), 2.0 * (2.0 * b.s * b.cout) * b.cin * double(n),
                                     b.convt->gemm_bytes() + double(n) * b.cin * 2 + double(n) * b.s * b.cout * 4,
                                     gemm_kernel_name(op)})))
                return rc;
        }
        n *= b.s;
        Tb *= b.s;
        const int C = b.cout;
        const int stage0 = 2 + 4 * static_cast<int>(bi);
        sink.stage(stage0, d.xa, size_t(n) * C);
        float* cur = d.xa;
        float* nxt = d.xb;
        for (int r = 0; r < 3; ++r) {
            const ResUnit& u = b.ru[r];
            const int dl = kDil[r];
            if (use_fused_unit(C, B, Tb, sms)) {
                // one fused kernel: snake1 -> dw -> snake2 -> pointwise -> + bias + x [-> Snake]
                ResUnitOp op;
                int epi = kResPlain;
                const float *sa = nullptr, *si = nullptr;
                void* y = nxt;
                double out_bytes = 4;
                if (r == 2 && !last_block) {
                    epi = kResSnakeF16;
                    sa = c->blocks[bi + 1].alpha.v;
                    si = c->blocks[bi + 1].alpha.inv;
                    y = d.s16;
                    out_bytes = 2;
                } else if (r == 2) {
                    // the final Snake, fp16 (the final conv's input, rounded as the
                    // reference's im2col + F16 mul_mat rounds it) into the fp32
                    // buffer's memory
                    epi = kResSnakeF16;
                    sa = c->final_alpha.v;
                    si = c->final_alpha.inv;
                    out_bytes = 2;
                }
                if ((rc = setup_resunit(&op, u.pw->dev, u.pw->type, C, dl, cur, y, epi, u.a1.v, u.a1.inv, u.dw,
                                        u.db.v, u.a2.v, u.a2.inv, u.pb.v, sa, si, B, Tb, sms, d.status)))
                    return rc;
                rc = sink.kernel([op](cudaStream_t s) { return op.launch(s); },
                                 {"resunit_b" + std::to_string(bi) + "u" + std::to_string(r),
                                  2.0 * C * C * double(n) + 20.0 * double(n) * C,
                                  u.pw->gemm_bytes() + double(n) * C * (4 + out_bytes), op.kernel_name()});
                if (rc) return rc;
                if (r < 2) sink.stage(stage0 + 1 + r, nxt, size_t(n) * C);
                std::swap(cur, nxt);
                continue;
            }
            {
                const float* x = cur;
                __half* h = d.h16;
                const int Bq = B, Tq = Tb;
                rc = sink.kernel(
                    [=](cudaStream_t s) {
                        return launch_res_pre(x, u.a1.v, u.a1.inv, u.dw, u.db.v, u.a2.v, u.a2.inv, h, C, Bq, Tq, dl,
                                              sms, s);
                    },
                    {"res_pre_b" + std::to_string(bi) + "u" + std::to_string(r), double(n) * C * 20.0,
                     double(n) * C * (4 + 2) + C * 11 * 4, res_pre_kernel_name(C, B, Tb, dl, 0, sms)});
                if (rc) return rc;
            }
            if (resunit_hg_fits(C) && int64_t(B) * ((Tb + kRuTT - 1) / kRuTT) >= sms) {
                // pointwise conv + bias + residual [-> Snake], tokens as M (all C channels in one tile)
                ResUnitOp op;
                int epi = kResPlain;
                const float *sa = nullptr, *si = nullptr;
                void* y = nxt;
                double out_bytes = 4;
                if (r == 2 && !last_block) {
                    epi = kResSnakeF16;
                    sa = c->blocks[bi + 1].alpha.v;
                    si = c->blocks[bi + 1].alpha.inv;
                    y = d.s16;
                    out_bytes = 2;
                } else if (r == 2) {
                    epi = kResSnakeF16;  // the final Snake, fp16 (the final conv's input)
                    sa = c->final_alpha.v;
                    si = c->final_alpha.inv;
                    out_bytes = 2;
                }
                if ((rc = setup_resunit(&op, u.pw->dev, u.pw->type, C, dl, cur, y, epi, u.a1.v, u.a1.inv, u.dw,
                                        u.db.v, u.a2.v, u.a2.inv, u.pb.v, sa, si, B, Tb, sms, d.status, d.h16)))
                    return rc;
                rc = sink.kernel([op](cudaStream_t s) { return op.launch(s); },
                                 {"pw_b" + std::to_string(bi) + "u" + std::to_string(r), 2.0 * C * C * double(n),
                                  u.pw->gemm_bytes() + double(n) * C * (2 + 4 + out_bytes), op.kernel_name()});
                if (rc) return rc;
                if (r < 2) sink.stage(stage0 + 1 + r, nxt, size_t(n) * C);
                std::swap(cur, nxt);
                continue;
            }
            GemmOp op;
            double out_bytes;
            if (r < 2) {
                rc = setup_pointwise(&op, u.pw->gemm_view(), C, C, d.h16, n, u.pb.v, cur, nullptr, nullptr, 0, nxt,
                                     d.status);
                out_bytes = 4;
            } else if (!last_block) {
                const Block& nb = c->blocks[bi + 1];
                rc = setup_pointwise(&op, u.pw->gemm_view(), C, C, d.h16, n, u.pb.v, cur, nb.alpha.v, nb.alpha.inv, 1,
                                     d.s16, d.status);
                out_bytes = 2;
            } else {
                // the final Snake, fp16 (the final conv's input)
                rc = setup_pointwise(&op, u.pw->gemm_view(), C, C, d.h16, n, u.pb.v, cur, c->final_alpha.v,
                                     c->final_alpha.inv, 1, nxt, d.status);
                out_bytes = 2;
            }
            if (rc) return rc;
            if ((rc = sink.gemm(op, {"pw_b" + std::to_string(bi) + "u" + std::to_string(r), 2.0 * C * C * double(n),
                                     u.pw->gemm_bytes() + double(n) * C * (2 + 4 + out_bytes), gemm_kernel_name(op)})))
                return rc;
            if (r < 2) sink.stage(stage0 + 1 + r, nxt, size_t(n) * C);
            std::swap(cur, nxt);
        }
        if (last_block) {
            // final conv over snake(x) (fp16, in `cur` after the swap)
            const __half* sx = reinterpret_cast<const __half*>(cur);
            float* o = d.out;
            const float* w = c->final_w;
            const float fb = c->final_bias;
            const int Tq = Tb, Bq = B;
            rc = sink.kernel(
                [=](cudaStream_t s) {
                    const int tt = final_tile(Bq, Tq, sms);
                    dim3 grid((Tq + tt - 1) / tt, Bq);
                    const cudaError_t e = launch_pdl(C == 96 ? final_kernel<96> : final_kernel<0>, grid, dim3(256),
                                                     final_smem_bytes(C, tt),
                                                     s, sx, w, fb, o, C, Tq, 0, tt);
                    return e == cudaSuccess ? VXB_OK : fail(VXB_ERR_BACKEND, "final launch");
                },
                {"final_conv", 14.0 * C * double(n), double(n) * C * 2 + double(n) * 4,
                 C == 96 ? "final_kernel<96>" : "final_kernel<0>"});
            if (rc) return rc;
        }
    }
    return VXB_OK;
}

// Records the launches into a plan (replayed later, optionally as a graph).
struct PlanSink : OpSink {
    Plan& P;
    explicit PlanSink(Plan& p) : P(p) {}
    int gemm(const GemmOp& op, OpInfo info) override {
        P.gemms.push_back(op);
        P.ops.push_back([&P = P, idx = P.gemms.size() - 1](cudaStream_t s) { return P.gemms[idx].launch(s); });
        P.info.push_back(std::move(info));
        return VXB_OK;
    }
    int kernel(std::function<int(cudaStream_t)> fn, OpInfo info) override {
        P.ops.push_back(std::move(fn));
        P.info.push_back(std::move(info));
        return VXB_OK;
    }
    void stage(int stage, float* buf, size_t floats) override { P.stage_buf[stage] = {buf, floats, P.ops.size() - 1}; }
};

// Binds the encoder weights (audio_vae.encoder.*, the names and layouts
// load_encoder_weights reads, src/audio-vae.cpp:331-363) and derives their
// fp32 vectors, the fp16 copies of Q4_0 matrices and the strided convs' /
// fc_mu's weights reordered to [Cout][K][Cin], once per vxb_prepare.
int bind_encoder(vxb_ctx* c) {
    if (c->enc_bound) return VXB_OK;
    const int E = c->encoder_dim, nb = static_cast<int>(c->enc_rates.size());
    if (E <= 0 || nb == 0) return fail(VXB_ERR_NOT_READY, "no encoder config (GGUF keys or vxb_set_encoder_config)");
    const std::string p = "audio_vae.encoder.";
    const DevTensor* w0 = get(c, p + "block.0.weight");
    if (!w0) return fail(VXB_ERR_MISSING_TENSOR, "missing tensor " + p + "block.0.weight");
    if (w0->nelem() != int64_t(7) * E)
        return fail(VXB_ERR_INVALID_FORMAT, "the model carries no encoder weights (placeholder encoder tensors)");
    // the head conv kernel gives each thread a quad of channels, 256 threads per block
    if (E % 32 || E > 1024) return fail(VXB_ERR_INVALID_FORMAT, "encoder width must be a multiple of 32 and <= 1024");
    int rc;
    if ((rc = derive_taps(c, p + "block.0.weight", E, &c->enc_w0))) return rc;
    if ((rc = derive_vec(c, p + "block.0.bias", E, false, &c->enc_b0))) return rc;
    c->enc_blocks.clear();
    int C = E;
    for (int bi = 0; bi < nb; ++bi) {
        EncBlock b;
        b.cin = C;
        b.cout = 2 * C;
        b.s = c->enc_rates[bi];
        // channel counts: 16-byte vectors in the elementwise kernels, TMA rows in the GEMMs
        if (C % 32) return fail(VXB_ERR_INVALID_FORMAT, "encoder channels must be multiples of 32");
        const std::string bp = p + "block." + std::to_string(bi + 1) + ".block.";
        for (int r = 0; r < 3; ++r) {
            const std::string rp = bp + std::to_string(r) + ".block.";
            ResUnit& u = b.ru[r];
            if ((rc = derive_vec(c, rp + "0.alpha", C, true, &u.a1))) return rc;
            if ((rc = derive_taps(c, rp + "1.weight", C, &u.dw))) return rc;
            if ((rc = derive_vec(c, rp + "1.bias", C, false, &u.db))) return rc;
            if ((rc = derive_vec(c, rp + "2.alpha", C, true, &u.a2))) return rc;
            if ((rc = check_matrix(c, rp + "3.weight", C, C, &u.pw))) return rc;
            if ((rc = derive_vec(c, rp + "3.bias", C, false, &u.pb))) return rc;
        }
        if ((rc = derive_vec(c, bp + "3.alpha", C, true, &b.alpha))) return rc;
        if ((rc = check_matrix(c, bp + "4.weight", int64_t(2) * b.s * C, b.cout, &b.conv))) return rc;
        if (!(b.conv->n_dims == 3 ? b.conv->ne[0] == 2 * b.s && b.conv->ne[1] == C : b.conv->ne[0] == 2 * b.s * C))
            return fail(VXB_ERR_INVALID_FORMAT, bp + "4.weight: expected [2s, Cin, Cout] or [2s*Cin, Cout]");
        if ((rc = derive_vec(c, bp + "4.bias", b.cout, false, &b.bias))) return rc;
        c->enc_blocks.push_back(b);
        C *= 2;
    }
    const int Lt = c->latent_dim;
    if ((rc = check_matrix(c, p + "fc_mu.weight", int64_t(3) * C, Lt, &c->fc_mu))) return rc;
    if (!(c->fc_mu->n_dims == 3 ? c->fc_mu->ne[0] == 3 && c->fc_mu->ne[1] == C : c->fc_mu->ne[0] == 3 * C))
        return fail(VXB_ERR_INVALID_FORMAT, "fc_mu.weight: expected [3, C, latent] or [3*C, latent]");
    if ((rc = derive_vec(c, p + "fc_mu.bias", Lt, false, &c->fc_b))) return rc;
    // conv weights reordered to [Cout][K][Cin]: an im2col row is then K whole input rows
    auto permute = [&](const DevTensor* t, int cout, int cin, int k, __half** out) {
        CUDA_TRY(cudaMalloc(out, sizeof(__half) * size_t(cout) * cin * k));
        c->derived_allocs.push_back(*out);
        permute_ck_kernel<<<grid_1d(int64_t(cout) * cin * k, 256), 256, 0, c->stream>>>(
            t->dev, t->type == VXB_TYPE_Q4_0 ? 1 : 0, *out, cout, cin, k);
        CUDA_TRY(cudaGetLastError());
        return VXB_OK;
    };
    for (EncBlock& b : c->enc_blocks)
        if ((rc = permute(b.conv, b.cout, b.cin, 2 * b.s, &b.wperm))) return rc;
    if ((rc = permute(c->fc_mu, Lt, C, 3, &c->fc_perm))) return rc;
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    c->enc_bound = true;
    return VXB_OK;
}

// Largest activation (floats) and largest im2col operand (halves) of an
// encode of B waveforms of T latent frames.
void enc_arena_sizes(const vxb_ctx* c, int B, int T, int64_t* max_x, int64_t* max_col) {
    int64_t L = int64_t(T) * vxb_encoder_hop(c);
    *max_x = int64_t(B) * L * c->encoder_dim;
    *max_col = 0;
    for (const EncBlock& b : c->enc_blocks) {
        const int64_t Lo = L / b.s;
        *max_col = std::max(*max_col, int64_t(B) * Lo * b.cin * 2 * b.s);
        *max_x = std::max(*max_x, int64_t(B) * L * b.cin);
        L = Lo;
        *max_x = std::max(*max_x, int64_t(B) * L * b.cout);
    }
    *max_col = std::max(*max_col, int64_t(B) * L * c->enc_blocks.back().cout * 3);
}

int launch_im2col(const __half* g, __half* col, int B, int L, int C, int K, int s, int lpad, int Lout,
                  cudaStream_t st) {
    const cudaError_t e = launch_pdl(im2col_rows_kernel, dim3(grid_1d(int64_t(B) * Lout * K * (C / 8), 256)),
                                     dim3(256), 0, st, g, col, B, L, C, K, s, lpad, Lout);
    return e == cudaSuccess ? VXB_OK : fail(VXB_ERR_BACKEND, std::string("im2col launch: ") + cudaGetErrorString(e));
}

// The launch sequence of one encode of B waveforms of T latent frames
// (T * hop samples each; encode_tensor, src/audio-vae.cpp:640-650):
//   head conv k7 -> per block: 3 residual units (the decoder's kernels: the
//   fused unit up to 128 channels, else prologue + pointwise GEMM), the last
//   one's epilogue applying the block's Snake and writing fp16 -> im2col
//   rows (k 2s, stride s, left pad 2 ceil(s/2)) -> the conv as one pointwise
//   GEMM (K = 2s Cin, weight in [Cout][2s][Cin] order) doubling the channels
//   (fp32, or fp16 after the last block: fc_mu's input)
//   -> fc_mu: im2col rows (k 3, left pad 2) -> GEMM -> transpose to [B][L][T].
int emit_encode(vxb_ctx* c, const DecodeBufs& d, int B, int T, OpSink& sink) {
    const int E = c->encoder_dim, Lt = c->latent_dim;
    const int sms = num_sms(c->device);
    int64_t L = int64_t(T) * vxb_encoder_hop(c);
    int rc;
    {
        const float *a = d.z, *w = c->enc_w0, *bb = c->enc_b0.v;
        float* o = d.xa;
        const int64_t n = int64_t(B) * L;
        const long long Lq = L;
        const int G = 256 / (E / 4);
        const int64_t runs = int64_t(B) * ((L + kHeadRun - 1) / kHeadRun);
        const int grid = static_cast<int>(std::min<int64_t>((runs + G - 1) / G, int64_t(sms) * 16));
        rc = sink.kernel(
            [=](cudaStream_t s) {
                const cudaError_t e = launch_pdl(enc_head_kernel, dim3(grid), dim3(256), 0, s, a, w, bb, o, B, Lq, E);
                return e == cudaSuccess ? VXB_OK : fail(VXB_ERR_BACKEND, "encoder head launch");
            },
            {"enc_head", 14.0 * double(n) * E, double(n) * (4 + E * 4), "enc_head_kernel"});
        if (rc) return rc;
    }
    float* cur = d.xa;
    float* nxt = d.xb;
    static const int kDil[3] = {1, 3, 9};
    const size_t nbk = c->enc_blocks.size();
    for (size_t bi = 0; bi < nbk; ++bi) {
        const EncBlock& b = c->enc_blocks[bi];
        const int C = b.cin;
        const int Lb = static_cast<int>(L);
        const int64_t n = int64_t(B) * L;
        const std::string tag = "enc_b" + std::to_string(bi);
        for (int r = 0; r < 3; ++r) {
            const ResUnit& u = b.ru[r];
            const int dl = kDil[r];
            const std::string nm = tag + "u" + std::to_string(r);
            // the last unit applies the block's Snake and writes fp16 (the conv's input)
            const bool last = r == 2;
            if (use_fused_unit(C, B, Lb, sms)) {
                ResUnitOp op;
                if ((rc = setup_resunit(&op, u.pw->dev, u.pw->type, C, dl, cur,
                                        last ? static_cast<void*>(d.g16) : nxt, last ? kResSnakeF16 : kResPlain,
                                        u.a1.v, u.a1.inv, u.dw, u.db.v, u.a2.v, u.a2.inv, u.pb.v,
                                        last ? b.alpha.v : nullptr, last ? b.alpha.inv : nullptr, B, Lb, sms,
                                        d.status)))
                    return rc;
                rc = sink.kernel([op](cudaStream_t s) { return op.launch(s); },
                                 {"resunit_" + nm, 2.0 * C * C * double(n) + 20.0 * double(n) * C,
                                  u.pw->gemm_bytes() + double(n) * C * (last ? 6 : 8), op.kernel_name()});
                if (rc) return rc;
                if (!last) std::swap(cur, nxt);
                continue;
            }
            {
                const float* x = cur;
                __half* h = d.h16;
                rc = sink.kernel(
                    [=](cudaStream_t s) {
                        return launch_res_pre(x, u.a1.v, u.a1.inv, u.dw, u.db.v, u.a2.v, u.a2.inv, h, C, B, Lb, dl,
                                              sms, s);
                    },
                    {"res_pre_" + nm, double(n) * C * 20.0, double(n) * C * (4 + 2) + C * 11 * 4,
                     res_pre_kernel_name(C, B, Lb, dl, 0, sms)});
                if (rc) return rc;
            }
            if (resunit_hg_fits(C) && int64_t(B) * ((Lb + kRuTT - 1) / kRuTT) >= sms) {
                // pointwise conv + bias + residual [-> Snake], tokens as M (all C channels in one tile)
                ResUnitOp op;
                if ((rc = setup_resunit(&op, u.pw->dev, u.pw->type, C, dl, cur,
                                        last ? static_cast<void*>(d.g16) : nxt, last ? kResSnakeF16 : kResPlain,
                                        u.a1.v, u.a1.inv, u.dw, u.db.v, u.a2.v, u.a2.inv, u.pb.v,
                                        last ? b.alpha.v : nullptr, last ? b.alpha.inv : nullptr, B, Lb, sms,
                                        d.status, d.h16)))
                    return rc;
                rc = sink.kernel([op](cudaStream_t s) { return op.launch(s); },
                                 {"pw_" + nm, 2.0 * C * C * double(n),
                                  u.pw->gemm_bytes() + double(n) * C * (last ? 8 : 10), op.kernel_name()});
                if (rc) return rc;
                if (!last) std::swap(cur, nxt);
                continue;
            }
            GemmOp op;
            if ((rc = setup_pointwise(&op, u.pw->gemm_view(), C, C, d.h16, n, u.pb.v, cur, last ? b.alpha.v : nullptr,
                                      last ? b.alpha.inv : nullptr, last ? 1 : 0,
                                      last ? static_cast<void*>(d.g16) : nxt, d.status)))
                return rc;
            if ((rc = sink.gemm(op, {"pw_" + nm, 2.0 * C * C * double(n),
                                     u.pw->gemm_bytes() + double(n) * C * (last ? 8 : 10), gemm_kernel_name(op)})))
                return rc;
            if (!last) std::swap(cur, nxt);
        }
        // im2col rows of the Snake output, then the strided conv as one GEMM
        const int K = 2 * b.s, lpad = 2 * ((b.s + 1) / 2);
        const int Lo = static_cast<int>((L + lpad - K) / b.s + 1);
        const int64_t no = int64_t(B) * Lo;
        {
            const __half* g = d.g16;
            __half* col = d.s16;
            const int s = b.s;
            rc = sink.kernel([=](cudaStream_t st) { return launch_im2col(g, col, B, Lb, C, K, s, lpad, Lo, st); },
                             {"im2col_" + tag, 0.0, double(n) * C * 2 + double(no) * C * K * 2, "im2col_rows_kernel"});
            if (rc) return rc;
        }
        // the last block writes fp16: fc_mu's im2col reads it
        const bool last_block = bi + 1 == nbk;
        GemmOp op;
        if ((rc = setup_pointwise(&op, WView{b.wperm, VXB_TYPE_F16, 0, nullptr, 0}, C * K, b.cout, d.s16, no,
                                  b.bias.v, nullptr, nullptr, nullptr, last_block ? 1 : 0,
                                  last_block ? static_cast<void*>(d.g16) : cur, d.status)))
            return rc;
        if ((rc = sink.gemm(op, {"conv_" + tag, 2.0 * b.cout * double(C) * K * double(no),
                                 b.conv->gemm_bytes() + double(no) * C * K * 2 + double(no) * b.cout * (last_block ? 2 : 4),
                                 gemm_kernel_name(op)})))
            return rc;
        L = Lo;
    }
    // fc_mu: conv k3 (left pad 2) -> [B*T][Lt], then the latent layout [B][Lt][T]
    const int C = c->enc_blocks.back().cout;
    const int64_t n = int64_t(B) * L;
    {
        const __half* g = d.g16;
        __half* col = d.s16;
        const int Lb = static_cast<int>(L);
        rc = sink.kernel([=](cudaStream_t st) { return launch_im2col(g, col, B, Lb, C, 3, 1, 2, Lb, st); },
                         {"im2col_fc_mu", 0.0, double(n) * C * 2 + double(n) * C * 3 * 2, "im2col_rows_kernel"});
        if (rc) return rc;
    }
    GemmOp op;
    if ((rc = setup_pointwise(&op, WView{c->fc_perm, VXB_TYPE_F16, 0, nullptr, 0}, C * 3, Lt, d.s16, n, c->fc_b.v,
                              nullptr, nullptr, nullptr, 0, nxt, d.status)))
        return rc;
    if ((rc = sink.gemm(op, {"conv_fc_mu", 2.0 * Lt * double(C) * 3 * double(n),
                             c->fc_mu->gemm_bytes() + double(n) * C * 3 * 2 + double(n) * Lt * 4, gemm_kernel_name(op)})))
        return rc;
    {
        const float* y = nxt;
        float* z = d.out;
        const int Tq = static_cast<int>(L);
        rc = sink.kernel(
            [=](cudaStream_t s) {
                const cudaError_t e = launch_pdl(latent_transpose_kernel, dim3(grid_1d(n * Lt, 256)), dim3(256), 0, s,
                                                 y, z, B, Tq, Lt);
                return e == cudaSuccess ? VXB_OK : fail(VXB_ERR_BACKEND, "latent transpose launch");
            },
            {"latent_transpose", 0.0, double(n) * Lt * 8, "latent_transpose_kernel"});
        if (rc) return rc;
    }
    return VXB_OK;
}

}  // namespace

extern "C" int vxb_build_plan(vxb_ctx* c, int B, int T, int use_graph) {
    if (!c || B <= 0 || T <= 0) return fail(VXB_ERR_INVALID_ARGUMENT, "bad plan shape");
    if (!c->prepared) return fail(VXB_ERR_NOT_READY, "call vxb_prepare before vxb_build_plan");
    DeviceGuard g(c->device);
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    if (c->plan) free_plan(c->plan.get());
    c->plan = std::make_unique<Plan>();
    Plan& P = *c->plan;
    P.B = B;
    P.T = T;
    P.use_graph = use_graph != 0;
    const int L = c->latent_dim, hop = vxb_hop(c);
    int64_t max_x, max_s;
    arena_sizes(c, B, T, &max_x, &max_s);
    CUDA_TRY(cudaMalloc(&P.z, sizeof(float) * B * L * T));
    CUDA_TRY(cudaMalloc(&P.out, sizeof(float) * int64_t(B) * T * hop));
    DecodeBufs& d = P.bufs;
    CUDA_TRY(cudaMalloc(&d.xa, sizeof(float) * max_x));
    CUDA_TRY(cudaMalloc(&d.xb, sizeof(float) * max_x));
    CUDA_TRY(cudaMalloc(&d.h16, sizeof(__half) * max_x));
    CUDA_TRY(cudaMalloc(&d.s16, sizeof(__half) * max_s));
    d.z = P.z;
    d.out = P.out;
    d.status = c->status;
    P.bytes = sizeof(float) * (B * L * T + int64_t(B) * T * hop + 2 * max_x) + sizeof(__half) * (max_x + max_s);
    PlanSink sink(P);
    int rc = emit_decode(c, d, B, T, sink);
    if (rc) return rc;
    if (P.use_graph) {
        CUDA_TRY(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        int orc = VXB_OK;
        cudaMemsetAsync(c->status, 0, sizeof(int), c->stream);
        for (auto& op : P.ops)
            if ((orc = op(c->stream))) break;
        cudaGraph_t graph = nullptr;
        cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
        if (orc) {
            if (graph) cudaGraphDestroy(graph);
            return orc;
        }
        if (e != cudaSuccess) return fail(VXB_ERR_BACKEND, std::string("graph capture: ") + cudaGetErrorString(e));
        P.graph = graph;
        CUDA_TRY(cudaGraphInstantiate(&P.exec, P.graph, 0));
    }
    return VXB_OK;
}

namespace {

int run_plan(vxb_ctx* c, cudaStream_t s) {
    Plan& P = *c->plan;
    if (P.use_graph) {
        CUDA_TRY(cudaGraphLaunch(P.exec, s));
    } else {
        CUDA_TRY(cudaMemsetAsync(c->status, 0, sizeof(int), s));
        for (auto& op : P.ops) {
            int rc = op(s);
            if (rc) return rc;
        }
    }
    return VXB_OK;
}

// Bounded wait for a stream: polls without sleeping for the first 2 ms (a
// streaming decode completes in well under that; a sleep would add the OS
// timer slack to every call), then sleeps between polls until the timeout.
int wait_stream(cudaStream_t s, int timeout_ms) {
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return VXB_OK;
        if (e != cudaErrorNotReady) return fail(VXB_ERR_BACKEND, std::string("stream: ") + cudaGetErrorString(e));
        const auto waited = std::chrono::steady_clock::now() - t0;
        if (waited > std::chrono::milliseconds(timeout_ms))
            return fail(VXB_ERR_TIMEOUT, "timed out waiting for the device");
        if (waited > std::chrono::milliseconds(2)) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

int check_status(vxb_ctx* c) {
    if (*c->status_host != 0)
        return fail(VXB_ERR_DEVICE_STATUS, "kernel bounded wait failed (code " + std::to_string(*c->status_host) + ")");
    return VXB_OK;
}

}  // namespace

extern "C" int vxb_decode(vxb_ctx* c, const float* z_host, float* out_host) {
    if (!c || !z_host || !out_host) return fail(VXB_ERR_INVALID_ARGUMENT, "null argument");
    if (!c->plan) return fail(VXB_ERR_NOT_READY, "no plan: call vxb_build_plan");
    DeviceGuard g(c->device);
    Plan& P = *c->plan;
    const size_t zin = sizeof(float) * P.B * c->latent_dim * P.T;
    const size_t zout = sizeof(float) * int64_t(P.B) * P.T * vxb_hop(c);
    CUDA_TRY(cudaMemcpyAsync(P.z, z_host, zin, cudaMemcpyHostToDevice, c->stream));
    int rc = run_plan(c, c->stream);
    if (rc) return rc;
    CUDA_TRY(cudaMemcpyAsync(out_host, P.out, zout, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaMemcpyAsync(c->status_host, c->status, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    if ((rc = wait_stream(c->stream, 60000))) return rc;
    return check_status(c);
}

extern "C" int vxb_decode_device(vxb_ctx* c, const float* z_dev, float* out_dev, void* stream) {
    if (!c || !z_dev || !out_dev) return fail(VXB_ERR_INVALID_ARGUMENT, "null argument");
    if (!c->plan) return fail(VXB_ERR_NOT_READY, "no plan: call vxb_build_plan");
    DeviceGuard g(c->device);
    Plan& P = *c->plan;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    const size_t zin = sizeof(float) * P.B * c->latent_dim * P.T;
    const size_t zout = sizeof(float) * int64_t(P.B) * P.T * vxb_hop(c);
    if (z_dev != P.z) CUDA_TRY(cudaMemcpyAsync(P.z, z_dev, zin, cudaMemcpyDeviceToDevice, s));
    int rc = run_plan(c, s);
    if (rc) return rc;
    if (out_dev != P.out) CUDA_TRY(cudaMemcpyAsync(out_dev, P.out, zout, cudaMemcpyDeviceToDevice, s));
    CUDA_TRY(cudaMemcpyAsync(c->status_host, c->status, sizeof(int), cudaMemcpyDeviceToHost, s));
    return VXB_OK;
}

extern "C" int vxb_build_encode_plan(vxb_ctx* c, int B, int T) {
    if (!c || B <= 0 || T <= 0) return fail(VXB_ERR_INVALID_ARGUMENT, "bad encode plan shape");
    if (!c->prepared) return fail(VXB_ERR_NOT_READY, "call vxb_prepare before vxb_build_encode_plan");
    DeviceGuard g(c->device);
    int rc = bind_encoder(c);
    if (rc) return rc;
    const int64_t hop = vxb_encoder_hop(c);
    if (int64_t(T) * hop > (int64_t(1) << 30) / c->encoder_dim)
        return fail(VXB_ERR_INVALID_ARGUMENT, "encode plan: waveform too long for one plan");
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    if (c->enc_plan) free_plan(c->enc_plan.get());
    c->enc_plan = std::make_unique<Plan>();
    Plan& P = *c->enc_plan;
    P.B = B;
    P.T = T;
    int64_t max_x, max_col;
    enc_arena_sizes(c, B, T, &max_x, &max_col);
    CUDA_TRY(cudaMalloc(&P.z, sizeof(float) * B * T * hop));                 // waveforms
    CUDA_TRY(cudaMalloc(&P.out, sizeof(float) * int64_t(B) * c->latent_dim * T));  // latents
    DecodeBufs& d = P.bufs;
    CUDA_TRY(cudaMalloc(&d.xa, sizeof(float) * max_x));
    CUDA_TRY(cudaMalloc(&d.xb, sizeof(float) * max_x));
    CUDA_TRY(cudaMalloc(&d.h16, sizeof(__half) * max_x));
    CUDA_TRY(cudaMalloc(&d.s16, sizeof(__half) * max_col));
    CUDA_TRY(cudaMalloc(&d.g16, sizeof(__half) * max_x));
    d.z = P.z;
    d.out = P.out;
    d.status = c->status;
    P.bytes = sizeof(float) * (int64_t(B) * T * hop + int64_t(B) * c->latent_dim * T + 2 * max_x) +
              sizeof(__half) * (2 * max_x + max_col);
    PlanSink sink(P);
    return emit_encode(c, d, B, T, sink);
}

namespace {

int run_ops(vxb_ctx* c, Plan& P, cudaStream_t s) {
    CUDA_TRY(cudaMemsetAsync(c->status, 0, sizeof(int), s));
    for (auto& op : P.ops)
        if (int rc = op(s)) return rc;
    return VXB_OK;
}

}  // namespace

extern "C" int vxb_encode(vxb_ctx* c, const float* audio_host, float* latent_host) {
    if (!c || !audio_host || !latent_host) return fail(VXB_ERR_INVALID_ARGUMENT, "null argument");
    if (!c->enc_plan) return fail(VXB_ERR_NOT_READY, "no encode plan: call vxb_build_encode_plan");
    DeviceGuard g(c->device);
    Plan& P = *c->enc_plan;
    const size_t ain = sizeof(float) * P.B * P.T * vxb_encoder_hop(c);
    const size_t lout = sizeof(float) * int64_t(P.B) * c->latent_dim * P.T;
    CUDA_TRY(cudaMemcpyAsync(P.z, audio_host, ain, cudaMemcpyHostToDevice, c->stream));
    int rc = run_ops(c, P, c->stream);
    if (rc) return rc;
    CUDA_TRY(cudaMemcpyAsync(latent_host, P.out, lout, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaMemcpyAsync(c->status_host, c->status, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    if ((rc = wait_stream(c->stream, 60000))) return rc;
    return check_status(c);
}

extern "C" int vxb_encode_device(vxb_ctx* c, const float* audio_dev, float* latent_dev, void* stream) {
    if (!c || !audio_dev || !latent_dev) return fail(VXB_ERR_INVALID_ARGUMENT, "null argument");
    if (!c->enc_plan) return fail(VXB_ERR_NOT_READY, "no encode plan: call vxb_build_encode_plan");
    DeviceGuard g(c->device);
    Plan& P = *c->enc_plan;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    const size_t ain = sizeof(float) * P.B * P.T * vxb_encoder_hop(c);
    const size_t lout = sizeof(float) * int64_t(P.B) * c->latent_dim * P.T;
    if (audio_dev != P.z) CUDA_TRY(cudaMemcpyAsync(P.z, audio_dev, ain, cudaMemcpyDeviceToDevice, s));
    int rc = run_ops(c, P, s);
    if (rc) return rc;
    if (latent_dev != P.out) CUDA_TRY(cudaMemcpyAsync(latent_dev, P.out, lout, cudaMemcpyDeviceToDevice, s));
    CUDA_TRY(cudaMemcpyAsync(c->status_host, c->status, sizeof(int), cudaMemcpyDeviceToHost, s));
    return VXB_OK;
}

extern "C" int vxb_sync(vxb_ctx* c, int timeout_ms) {
    if (!c) return fail(VXB_ERR_INVALID_ARGUMENT, "null ctx");
    DeviceGuard g(c->device);
    int rc = wait_stream(c->stream, timeout_ms);
    if (rc) return rc;
    CUDA_TRY(cudaDeviceSynchronize());
    return check_status(c);
}

extern "C" int vxb_debug_stage(vxb_ctx* c, int stage, float* host_out, size_t n) {
    if (!c || !c->plan || !host_out) return fail(VXB_ERR_INVALID_ARGUMENT, "bad arguments");
    auto it = c->plan->stage_buf.find(stage);
    if (it == c->plan->stage_buf.end()) return fail(VXB_ERR_INVALID_ARGUMENT, "stage not materialised");
    const Plan::StageRef& ref = it->second;
    if (n < ref.floats) return fail(VXB_ERR_INVALID_ARGUMENT, "host buffer too small");
    DeviceGuard g(c->device);
    // Later stages reuse the buffer, so re-run the launch list up to the op
    // that writes this stage (on the latent still resident from the last decode).
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    CUDA_TRY(cudaMemsetAsync(c->status, 0, sizeof(int), c->stream));
    for (size_t i = 0; i <= ref.last_op && i < c->plan->ops.size(); ++i) {
        int rc = c->plan->ops[i](c->stream);
        if (rc) return rc;
    }
    CUDA_TRY(cudaMemcpyAsync(host_out, ref.buf, ref.floats * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaMemcpyAsync(c->status_host, c->status, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    int rc = wait_stream(c->stream, 60000);
    if (rc) return rc;
    return check_status(c);
}

extern "C" int vxb_debug_wait_probe(vxb_ctx* c, int limit_us, void* stream) {
    if (!c || limit_us < 1 || limit_us > 2000000) return fail(VXB_ERR_INVALID_ARGUMENT, "wait probe: bad limit");
    DeviceGuard g(c->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    CUDA_TRY(cudaMemsetAsync(c->status, 0, sizeof(int), s));
    wait_probe_kernel<<<1, 32, 0, s>>>(c->status, static_cast<unsigned long long>(limit_us) * 1000ull);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaMemcpyAsync(c->status_host, c->status, sizeof(int), cudaMemcpyDeviceToHost, s));
    return VXB_OK;
}

// ------------------------------------------------------ single-kernel APIs --

extern "C" int vxb_q4_0_dequant(const void* blocks, int64_t n, float* out, void* stream) {
    if (!blocks || !out || n <= 0 || n % 32) return fail(VXB_ERR_INVALID_ARGUMENT, "bad dequant arguments");
    q4_0_dequant_kernel<<<grid_1d(n / 32, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(blocks), out, n / 32);
    CUDA_TRY(cudaGetLastError());
    return VXB_OK;
}

extern "C" int vxb_snake(const float* x, const float* alpha, int C, int64_t N, float* y, void* stream) {
    if (!x || !alpha || !y || C <= 0 || N <= 0) return fail(VXB_ERR_INVALID_ARGUMENT, "bad snake arguments");
    snake_kernel<<<grid_1d(N * C, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, alpha, nullptr, y, C,
                                                                                       N * C);
    CUDA_TRY(cudaGetLastError());
    return VXB_OK;
}

namespace {

// Unit entry points receive the GGUF bytes as they are; a Q4_0 weight gets a
// stream-ordered split copy (nibbles + scales), freed after the launch.
struct PaddedQ4 {
    SplitQ4 q4;
    cudaStream_t s = nullptr;
    ~PaddedQ4() {
        if (q4.q) cudaFreeAsync(q4.q, s);
        if (q4.s) cudaFreeAsync(q4.s, s);
    }
};

int view_for(const void* w, int w_type, int64_t inner, int64_t rows, cudaStream_t st, PaddedQ4* tmp, WView* out) {
    *out = WView{w, w_type, 0, nullptr, 0};
    if (w_type != VXB_TYPE_Q4_0) return VXB_OK;
    tmp->s = st;
    int rc = split_q4(w, inner, rows, st, true, &tmp->q4);
    if (rc) return rc;
    *out = WView{tmp->q4.q, w_type, tmp->q4.pitch, tmp->q4.s, tmp->q4.spitch};
    return VXB_OK;
}

}  // namespace

extern "C" int vxb_pointwise(const void* w, int w_type, int K, int M, const void* x_f16, int64_t N,
                             const float* bias, const float* res, const float* snake_alpha, int out_f16, void* y,
                             void* stream) {
    if (!w || !x_f16 || !bias || !y) return fail(VXB_ERR_INVALID_ARGUMENT, "null argument");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    PaddedQ4 tmp;
    WView wv;
    int rc = view_for(w, w_type, K, M, st, &tmp, &wv);
    if (rc) return rc;
    GemmOp op;
    rc = setup_pointwise(&op, wv, K, M, x_f16, N, bias, res, snake_alpha, nullptr, out_f16, y, nullptr);
    if (rc) return rc;
    return op.launch(st);
}

namespace {

// Stream-ordered scratch for the unit entry points, freed when it goes out of scope.
struct Scratch {
    std::vector<void*> p;
    cudaStream_t s;
    explicit Scratch(cudaStream_t st) : s(st) {}
    ~Scratch() {
        for (void* q : p) cudaFreeAsync(q, s);
    }
    template <typename T>
    int get(size_t n, T** out) {
        void* q = nullptr;
        CUDA_TRY(cudaMallocAsync(&q, sizeof(T) * std::max<size_t>(n, 1), s));
        p.push_back(q);
        *out = static_cast<T*>(q);
        return VXB_OK;
    }
};

// 1 / (alpha + 1e-9) on the device (the reference's derived Snake vector).
int inv_of(const float* alpha, int C, Scratch& sc, float** inv) {
    int rc = sc.get(size_t(C), inv);
    if (rc) return rc;
    float* copy = nullptr;
    if ((rc = sc.get(size_t(C), &copy))) return rc;
    vec_to_f32_kernel<<<grid_1d(C, 256), 256, 0, sc.s>>>(alpha, VXB_TYPE_F32, C, copy, *inv);
    CUDA_TRY(cudaGetLastError());
    return VXB_OK;
}

}  // namespace

extern "C" int vxb_residual_unit(const void* w, int w_type, int C, int d, const float* x, int batch, int T,
                                 const float* a1, const float* dw, const float* db, const float* a2,
                                 const float* pb, const float* out_alpha, int out_f16, void* y, void* stream) {
    if (!w || !x || !a1 || !dw || !db || !a2 || !pb || !y || C <= 0 || batch <= 0 || T <= 0 || d < 1 || d > 9)
        return fail(VXB_ERR_INVALID_ARGUMENT, "residual unit: bad arguments");
    if (C % 8) return fail(VXB_ERR_INVALID_ARGUMENT, "residual unit: C must be a multiple of 8");
    if (out_f16 && !out_alpha) return fail(VXB_ERR_INVALID_ARGUMENT, "residual unit: fp16 output needs a Snake");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    const int sms = num_sms(dev);
    Scratch sc(st);
    float *i1 = nullptr, *i2 = nullptr, *io = nullptr;
    int rc = inv_of(a1, C, sc, &i1);
    if (!rc) rc = inv_of(a2, C, sc, &i2);
    if (!rc && out_alpha) rc = inv_of(out_alpha, C, sc, &io);
    if (rc) return rc;
    const int epi = !out_alpha ? kResPlain : (out_f16 ? kResSnakeF16 : kResSnakeF32);
    const int64_t N = int64_t(batch) * T;
    ResUnitOp op;
    if (resunit_fits(C)) {
        if ((rc = setup_resunit(&op, w, w_type, C, d, x, y, epi, a1, i1, dw, db, a2, i2, pb, out_alpha, io, batch,
                                T, sms, nullptr)))
            return rc;
        return op.launch(st);
    }
    __half* h = nullptr;
    if ((rc = sc.get(size_t(N) * C, &h))) return rc;
    if ((rc = launch_res_pre(x, a1, i1, dw, db, a2, i2, h, C, batch, T, d, sms, st))) return rc;
    if (resunit_hg_fits(C) && int64_t(batch) * ((T + kRuTT - 1) / kRuTT) >= sms) {
        if ((rc = setup_resunit(&op, w, w_type, C, d, x, y, epi, a1, i1, dw, db, a2, i2, pb, out_alpha, io, batch,
                                T, sms, nullptr, h)))
            return rc;
        return op.launch(st);
    }
    PaddedQ4 tmp;
    WView wv;
    if ((rc = view_for(w, w_type, C, C, st, &tmp, &wv))) return rc;
    GemmOp g;
    if ((rc = setup_pointwise(&g, wv, C, C, h, N, pb, x, out_alpha, io, out_f16, y, nullptr))) return rc;
    return g.launch(st);
}

extern "C" int vxb_convt(const void* w, int w_type, int Cin, int Cout, int s, const void* x_f16, int B, int T,
                         const float* bias, float* y, void* stream) {
    if (!w || !x_f16 || !bias || !y) return fail(VXB_ERR_INVALID_ARGUMENT, "null argument");
    if (s <= 0 || Cout <= 0 || Cin <= 0) return fail(VXB_ERR_INVALID_ARGUMENT, "convt: bad extents");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    PaddedQ4 tmp;
    WView wv;
    int rc = view_for(w, w_type, int64_t(2) * s * Cout, Cin, st, &tmp, &wv);
    if (rc) return rc;
    GemmOp op;
    rc = setup_convt(&op, wv, Cin, Cout, s, x_f16, B, T, bias, y, nullptr);
    if (rc) return rc;
    return op.launch(st);
}

// ------------------------------------------------------------ introspection --

namespace {

const Plan* plan_of(const vxb_ctx* c, int which) {
    if (!c) return nullptr;
    return which == 1 ? c->enc_plan.get() : c->plan.get();
}

int op_info(const Plan* P, int idx, char* name, int name_cap, char* kernel, int kernel_cap, double* flops,
            double* bytes) {
    if (!P || idx < 0 || idx >= static_cast<int>(P->info.size())) return fail(VXB_ERR_INVALID_ARGUMENT, "bad op index");
    const auto& in = P->info[idx];
    if (name && name_cap > 0) std::snprintf(name, name_cap, "%s", in.name.c_str());
    if (kernel && kernel_cap > 0) std::snprintf(kernel, kernel_cap, "%s", in.kernel.c_str());
    if (flops) *flops = in.flops;
    if (bytes) *bytes = in.bytes;
    return VXB_OK;
}

// Device time of every op of a plan (CUDA events between launches on the
// context's stream), averaged over reps, the buffer `flush` rewritten
// before each rep.
int time_plan_ops(vxb_ctx* c, Plan& P, int reps, void* flush, size_t flush_bytes, float* ms_out) {
    DeviceGuard g(c->device);
    const size_t nops = P.ops.size();
    std::vector<cudaEvent_t> ev(nops + 1);
    for (auto& e : ev) CUDA_TRY(cudaEventCreate(&e));
    std::vector<double> acc(nops, 0.0);
    int rc = VXB_OK;
    for (int r = 0; r < reps && rc == VXB_OK; ++r) {
        if (flush && flush_bytes) CUDA_TRY(cudaMemsetAsync(flush, r & 0xff, flush_bytes, c->stream));
        CUDA_TRY(cudaMemsetAsync(c->status, 0, sizeof(int), c->stream));
        CUDA_TRY(cudaEventRecord(ev[0], c->stream));
        for (size_t i = 0; i < nops && rc == VXB_OK; ++i) {
            rc = P.ops[i](c->stream);
            CUDA_TRY(cudaEventRecord(ev[i + 1], c->stream));
        }
        CUDA_TRY(cudaMemcpyAsync(c->status_host, c->status, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
        if (rc == VXB_OK) rc = wait_stream(c->stream, 60000);
        for (size_t i = 0; i < nops && rc == VXB_OK; ++i) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
            acc[i] += ms;
        }
    }
    for (auto& e : ev) cudaEventDestroy(e);
    if (rc) return rc;
    for (size_t i = 0; i < nops; ++i) ms_out[i] = static_cast<float>(acc[i] / reps);
    return check_status(c);
}

}  // namespace

extern "C" int vxb_plan_num_ops(const vxb_ctx* c) {
    return (c && c->plan) ? static_cast<int>(c->plan->ops.size()) : 0;
}

extern "C" int vxb_plan_op_info(const vxb_ctx* c, int idx, char* name, int name_cap, char* kernel, int kernel_cap,
                                double* flops, double* bytes) {
    return op_info(plan_of(c, 0), idx, name, name_cap, kernel, kernel_cap, flops, bytes);
}

extern "C" int vxb_time_ops(vxb_ctx* c, int reps, void* flush, size_t flush_bytes, float* ms_out) {
    if (!c || !c->plan || reps <= 0 || !ms_out) return fail(VXB_ERR_INVALID_ARGUMENT, "bad arguments");
    return time_plan_ops(c, *c->plan, reps, flush, flush_bytes, ms_out);
}

extern "C" int vxb_encode_num_ops(const vxb_ctx* c) {
    return (c && c->enc_plan) ? static_cast<int>(c->enc_plan->ops.size()) : 0;
}

extern "C" int vxb_encode_op_info(const vxb_ctx* c, int idx, char* name, int name_cap, char* kernel, int kernel_cap,
                                  double* flops, double* bytes) {
    return op_info(plan_of(c, 1), idx, name, name_cap, kernel, kernel_cap, flops, bytes);
}

extern "C" int vxb_encode_time_ops(vxb_ctx* c, int reps, void* flush, size_t flush_bytes, float* ms_out) {
    if (!c || !c->enc_plan || reps <= 0 || !ms_out) return fail(VXB_ERR_INVALID_ARGUMENT, "bad arguments");
    return time_plan_ops(c, *c->enc_plan, reps, flush, flush_bytes, ms_out);
}

// ------------------------------------------------ allocation-free decode --
//
// vxb_decode_static runs the same kernels as a planned decode, but every
// intermediate activation lives in the fixed device array below instead of
// a plan arena, so the call itself allocates nothing.

namespace {

// Scratch for vxb_decode_static: two fp32 activation buffers, two fp16
// GEMM-operand buffers and the device status word.  kStaticFrames latent
// frames (B*T) of the VoxCPM decoder (1536 channels, rates 8,8,5,2) need
// 720 KiB each, so the array is 5.63 MiB.  It lives as long as the library
// is loaded, on every GPU that loads it.
constexpr int kStaticFrames = 8;
constexpr size_t kStaticActFloats = size_t(61440) * kStaticFrames;  // largest stage, floats
constexpr size_t kStaticBytes = 2 * kStaticActFloats * sizeof(float) + 2 * kStaticActFloats * sizeof(__half) + 256;
static __device__ __align__(256) uint8_t g_static_scratch[kStaticBytes];

// Device address of g_static_scratch per device, looked up once (with that
// device current) under a per-device once_flag, so host threads that make
// their first call on one device at the same time do not race.  In host
// code the symbol is only a host-side stand-in, never a device pointer.
uint8_t* g_static_ptr[64] = {};
cudaError_t g_static_err[64] = {};
std::once_flag g_static_once[64];

int static_scratch(int dev, uint8_t** out) {
    if (dev < 0 || dev >= 64) return fail(VXB_ERR_BACKEND, "device index out of range");
    std::call_once(g_static_once[dev], [dev] {
        void* p = nullptr;
        g_static_err[dev] = cudaGetSymbolAddress(&p, g_static_scratch);
        if (g_static_err[dev] == cudaSuccess) g_static_ptr[dev] = static_cast<uint8_t*>(p);
    });
    if (g_static_err[dev] != cudaSuccess)
        return fail(VXB_ERR_BACKEND, std::string("cudaGetSymbolAddress(static scratch): ") +
                                         cudaGetErrorString(g_static_err[dev]));
    *out = g_static_ptr[dev];
    return VXB_OK;
}

// Launches every op as soon as it is emitted.
struct LaunchSink : OpSink {
    cudaStream_t s;
    explicit LaunchSink(cudaStream_t st) : s(st) {}
    int gemm(const GemmOp& op, OpInfo) override { return op.launch(s); }
    int kernel(std::function<int(cudaStream_t)> fn, OpInfo) override { return fn(s); }
};

}  // namespace

extern "C" int vxb_decode_static(vxb_ctx* c, const float* z_dev, float* out_dev, int B, int T, void* stream) {
    if (!c || !z_dev || !out_dev || B <= 0 || T <= 0) return fail(VXB_ERR_INVALID_ARGUMENT, "bad arguments");
    if (!c->prepared) return fail(VXB_ERR_NOT_READY, "call vxb_prepare first");
    int64_t max_x, max_s;
    arena_sizes(c, B, T, &max_x, &max_s);
    if (max_x > int64_t(kStaticActFloats) || max_s > int64_t(kStaticActFloats))
        return fail(VXB_ERR_INVALID_ARGUMENT,
                    "vxb_decode_static: shape needs " + std::to_string(std::max(max_x, max_s)) +
                        " activation elements, the static scratch holds " + std::to_string(kStaticActFloats) +
                        " (B*T <= " + std::to_string(kStaticFrames) + " frames for the VoxCPM decoder)");
    DeviceGuard g(c->device);
    uint8_t* base = nullptr;
    int rc = static_scratch(c->device, &base);
    if (rc) return rc;
    DecodeBufs d;
    d.z = z_dev;
    d.out = out_dev;
    d.xa = reinterpret_cast<float*>(base);
    d.xb = d.xa + kStaticActFloats;
    d.h16 = reinterpret_cast<__half*>(d.xb + kStaticActFloats);
    d.s16 = d.h16 + kStaticActFloats;
    d.status = reinterpret_cast<int*>(d.s16 + kStaticActFloats);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    CUDA_TRY(cudaMemsetAsync(d.status, 0, sizeof(int), s));  // the status word must start at zero
    LaunchSink sink(s);
    if ((rc = emit_decode(c, d, B, T, sink))) return rc;
    // report a failed bounded wait through vxb_sync (pinned word made at vxb_open)
    CUDA_TRY(cudaMemcpyAsync(c->status_host, d.status, sizeof(int), cudaMemcpyDeviceToHost, s));
    return VXB_OK;
}

// ------------------------------------------------------- stateful streaming --
//
// A vxb_stream decodes one latent stream n frames per push and carries every
// causal layer's left context from push to push: each layer reads a window
// [history rows | this push's rows] of its own input -- 6 latent frames for
// model.0, 1 input row for each transposed conv, 6*d rows for each residual
// unit's dilated conv, 6 rows for the final conv -- and computes only the
// new rows.  The history of a fresh stream is zero, which is exactly the
// causal zero padding of a sequence start, so the pushes together emit the
// continuous decode of the whole stream.  Two window sets alternate between
// pushes (one CUDA graph each); the end of a push copies the tail of every
// window of the set in use into the head of the other set's window.

namespace {

// One strided copy of the shift: `count` segments of `words` 32-bit words.
struct ShiftSeg {
    const uint32_t* src;
    uint32_t* dst;
    int count, words;
    int src_stride, dst_stride;  // in words
};

__global__ void shift_history_kernel(const ShiftSeg* __restrict__ segs, int nseg) {
    for (int g = blockIdx.x; g < nseg; g += gridDim.x) {
        const ShiftSeg sg = segs[g];
        const int total = sg.count * sg.words;
        for (int i = threadIdx.x; i < total; i += blockDim.x) {
            const int k = i / sg.words, w = i - k * sg.words;
            sg.dst[k * sg.dst_stride + w] = sg.src[k * sg.src_stride + w];
        }
    }
}

// The windows of one set.
struct StreamSet {
    float* z = nullptr;                 // [L][6 + n]: the latent window, t fastest per channel
    std::vector<__half*> wc;            // per block: transposed-conv input [1 + n_b][Cin] (fp16, Snake applied)
    std::vector<std::array<float*, 3>> wx;  // per block and unit: residual-stream window [6d + m_b][Cout] (fp32)
    __half* wf = nullptr;               // final conv input [6 + m_last][C_last] (fp16, final Snake applied)
    ShiftSeg* segs = nullptr;           // device copy of the shift into the other set
    int nseg = 0;
    Plan plan;                          // ops + graph of a push on this set
};

}  // namespace

struct vxb_stream {
    vxb_ctx* c = nullptr;
    int n = 0;                          // latent frames per push
    int parity = 0;                     // set used by the next push
    StreamSet set[2];
    __half* h0 = nullptr;               // model.0 output [n][L]
    __half* h = nullptr;                // prologue output [m_max][C_max]
    float* out = nullptr;               // [n * hop]
    std::vector<void*> allocs;
    std::vector<std::pair<void*, size_t>> wins;  // every window of both sets (zeroed by a reset)
};

namespace {

int stream_alloc(vxb_stream* st, size_t bytes, void** p) {
    CUDA_TRY(cudaMalloc(p, std::max<size_t>(bytes, 16)));
    st->allocs.push_back(*p);
    return VXB_OK;
}

// The launches of one push on window set p (and the shift into set 1 - p).
int emit_stream_push(vxb_stream* st, int p, OpSink& sink) {
    vxb_ctx* c = st->c;
    StreamSet& S = st->set[p];
    StreamSet& O = st->set[1 - p];
    const int L = c->latent_dim, D = c->decoder_dim, n = st->n;
    int* status = c->status;
    static const int kDil[3] = {1, 3, 9};
    const int sms = num_sms(c->device);
    int rc;
    std::vector<ShiftSeg> segs;
    auto seg_rows = [&](const void* src_win, void* dst_win, int64_t hist_row0, int64_t rows, int64_t cols, int elem) {
        const int64_t words = rows * cols * elem / 4;
        segs.push_back({static_cast<const uint32_t*>(src_win) + hist_row0 * cols * elem / 4,
                        static_cast<uint32_t*>(dst_win), 1, static_cast<int>(words), 0, 0});
    };
    {   // model.0 over the latent window (6 history frames), model.1 into block 0's window (row 1)
        const float* z = S.z;
        const float *w = c->dw0, *bb = c->b0.v;
        __half* o = st->h0;
        rc = sink.kernel(
            [=](cudaStream_t s) {
                const cudaError_t e = launch_pdl(head_kernel, dim3(grid_1d(int64_t(n) * L, 256)), dim3(256), 0, s, z, w,
                                                 bb, o, 1, L, n + 6, 6);
                return e == cudaSuccess ? VXB_OK : fail(VXB_ERR_BACKEND, "head launch");
            },
            {"head_dw", 14.0 * n * L, double(n) * L * 6, "head_kernel"});
        if (rc) return rc;
        segs.push_back({reinterpret_cast<const uint32_t*>(S.z) + n, reinterpret_cast<uint32_t*>(O.z), L, 6, n + 6, n + 6});
        GemmOp op;
        const Block& b0 = c->blocks[0];
        if ((rc = setup_pointwise(&op, c->pw1->gemm_view(), L, D, st->h0, n, c->b1.v, nullptr, b0.alpha.v,
                                  b0.alpha.inv, 1, S.wc[0] + D, status)))
            return rc;
        if ((rc = sink.gemm(op, {"pw_model1", 2.0 * D * L * n, c->pw1->gemm_bytes(), gemm_kernel_name(op)}))) return rc;
    }
    int64_t nb = n;  // this push's input frames of the block
    const size_t nblk = c->blocks.size();
    for (size_t bi = 0; bi < nblk; ++bi) {
        const Block& b = c->blocks[bi];
        const bool last_block = bi + 1 == nblk;
        const int C = b.cout;
        const int64_t m = nb * b.s;  // this push's output rows of the block
        {
            GemmOp op;
            if ((rc = setup_convt(&op, b.convt->gemm_view(), b.cin, C, b.s, S.wc[bi], 1, static_cast<int>(1 + nb),
                                  b.bias.v, S.wx[bi][0] + 6 * int64_t(C), status, 1)))
                return rc;
            if ((rc = sink.gemm(op, {"convt_b" + std::to_string(bi), 2.0 * (2.0 * b.s * C) * b.cin * double(nb),
                                     b.convt->gemm_bytes(), gemm_kernel_name(op)})))
                return rc;
            seg_rows(S.wc[bi], O.wc[bi], nb, 1, b.cin, 2);
        }
        for (int r = 0; r < 3; ++r) {
            const ResUnit& u = b.ru[r];
            const int dl = kDil[r];
            float* x = S.wx[bi][r];  // [6 dl + m][C]
            {
                __half* hh = st->h;
                const int mq = static_cast<int>(m);
                rc = sink.kernel(
                    [=](cudaStream_t s) {
                        return launch_res_pre(x, u.a1.v, u.a1.inv, u.dw, u.db.v, u.a2.v, u.a2.inv, hh, C, 1, mq, dl,
                                              sms, s, 6 * dl);
                    },
                    {"res_pre_b" + std::to_string(bi) + "u" + std::to_string(r), double(m) * C * 20.0,
                     double(m) * C * 6, res_pre_kernel_name(C, 1, static_cast<int>(m), dl, 6 * dl, sms)});
                if (rc) return rc;
            }
            GemmOp op;
            const float* res = x + 6 * dl * int64_t(C);
            if (r < 2) {
                rc = setup_pointwise(&op, u.pw->gemm_view(), C, C, st->h, m, u.pb.v, res, nullptr, nullptr, 0,
                                     S.wx[bi][r + 1] + 6 * kDil[r + 1] * int64_t(C), status);
            } else if (!last_block) {
                const Block& nbk = c->blocks[bi + 1];
                rc = setup_pointwise(&op, u.pw->gemm_view(), C, C, st->h, m, u.pb.v, res, nbk.alpha.v, nbk.alpha.inv, 1,
                                     S.wc[bi + 1] + C, status);
            } else {
                rc = setup_pointwise(&op, u.pw->gemm_view(), C, C, st->h, m, u.pb.v, res, c->final_alpha.v,
                                     c->final_alpha.inv, 1, S.wf + 6 * int64_t(C), status);
            }
            if (rc) return rc;
            if ((rc = sink.gemm(op, {"pw_b" + std::to_string(bi) + "u" + std::to_string(r), 2.0 * C * C * double(m),
                                     u.pw->gemm_bytes(), gemm_kernel_name(op)})))
                return rc;
            seg_rows(x, O.wx[bi][r], m, 6 * dl, C, 4);
        }
        if (last_block) {
            const __half* sx = S.wf;
            float* o = st->out;
            const float* w = c->final_w;
            const float fb = c->final_bias;
            const int Tq = static_cast<int>(m);
            rc = sink.kernel(
                [=](cudaStream_t s) {
                    const int tt = final_tile(1, Tq, sms);
                    dim3 grid((Tq + tt - 1) / tt, 1);
                    const cudaError_t e = launch_pdl(C == 96 ? final_kernel<96> : final_kernel<0>, grid, dim3(256),
                                                     final_smem_bytes(C, tt), s,
                                                     sx, w, fb, o, C, Tq, 6, tt);
                    return e == cudaSuccess ? VXB_OK : fail(VXB_ERR_BACKEND, "final launch");
                },
                {"final_conv", 14.0 * C * double(m), double(m) * C * 2,
                 C == 96 ? "final_kernel<96>" : "final_kernel<0>"});
            if (rc) return rc;
            seg_rows(S.wf, O.wf, m, 6, C, 2);
        }
        nb = m;
    }
    // the shift: every window's tail -> the other set's head
    S.nseg = static_cast<int>(segs.size());
    CUDA_TRY(cudaMalloc(&S.segs, sizeof(ShiftSeg) * segs.size()));
    st->allocs.push_back(S.segs);
    CUDA_TRY(cudaMemcpy(S.segs, segs.data(), sizeof(ShiftSeg) * segs.size(), cudaMemcpyHostToDevice));
    const ShiftSeg* sg = S.segs;
    const int ns = S.nseg;
    return sink.kernel(
        [=](cudaStream_t s) {
            shift_history_kernel<<<ns, 256, 0, s>>>(sg, ns);
            const cudaError_t e = cudaGetLastError();
            return e == cudaSuccess ? VXB_OK : fail(VXB_ERR_BACKEND, "history shift launch");
        },
        {"shift_history", 0.0, 0.0, "shift_history_kernel"});
}

void free_stream(vxb_stream* st) {
    for (int p = 0; p < 2; ++p) {
        if (st->set[p].plan.exec) cudaGraphExecDestroy(st->set[p].plan.exec);
        if (st->set[p].plan.graph) cudaGraphDestroy(st->set[p].plan.graph);
    }
    for (void* q : st->allocs) cudaFree(q);
    st->allocs.clear();
}

// A fresh stream: every window of both sets zero (the causal zero padding of a
// sequence start), the next push on set 0.
int stream_zero(vxb_stream* st, cudaStream_t s) {
    for (auto& w : st->wins) CUDA_TRY(cudaMemsetAsync(w.first, 0, w.second, s));
    st->parity = 0;
    return VXB_OK;
}

}  // namespace

extern "C" int vxb_stream_open(vxb_ctx* c, int n, vxb_stream** out) {
    if (!c || !out || n <= 0 || n > 4096) return fail(VXB_ERR_INVALID_ARGUMENT, "vxb_stream_open: bad arguments");
    *out = nullptr;
    if (!c->prepared) return fail(VXB_ERR_NOT_READY, "call vxb_prepare before vxb_stream_open");
    DeviceGuard g(c->device);
    auto st = std::make_unique<vxb_stream>();
    st->c = c;
    st->n = n;
    const int L = c->latent_dim, nb_blocks = static_cast<int>(c->blocks.size());
    static const int kDil[3] = {1, 3, 9};
    int rc;
    auto& wins = st->wins;
    int64_t m_max = 1, cmax = 1;
    for (int p = 0; p < 2; ++p) {
        StreamSet& S = st->set[p];
        void* q = nullptr;
        if ((rc = stream_alloc(st.get(), sizeof(float) * L * (6 + n), &q))) { free_stream(st.get()); return rc; }
        S.z = static_cast<float*>(q);
        wins.push_back({q, sizeof(float) * L * (6 + n)});
        int64_t nb = n;
        S.wc.resize(nb_blocks);
        S.wx.resize(nb_blocks);
        for (int bi = 0; bi < nb_blocks; ++bi) {
            const Block& b = c->blocks[bi];
            const size_t wcb = sizeof(__half) * (1 + nb) * b.cin;
            if ((rc = stream_alloc(st.get(), wcb, &q))) { free_stream(st.get()); return rc; }
            S.wc[bi] = static_cast<__half*>(q);
            wins.push_back({q, wcb});
            const int64_t m = nb * b.s;
            for (int r = 0; r < 3; ++r) {
                const size_t wxb = sizeof(float) * (6 * kDil[r] + m) * b.cout;
                if ((rc = stream_alloc(st.get(), wxb, &q))) { free_stream(st.get()); return rc; }
                S.wx[bi][r] = static_cast<float*>(q);
                wins.push_back({q, wxb});
            }
            m_max = std::max(m_max, m);
            cmax = std::max<int64_t>(cmax, b.cout);
            nb = m;
        }
        const size_t wfb = sizeof(__half) * (6 + nb) * c->blocks.back().cout;
        if ((rc = stream_alloc(st.get(), wfb, &q))) { free_stream(st.get()); return rc; }
        S.wf = static_cast<__half*>(q);
        wins.push_back({q, wfb});
    }
    void* q = nullptr;
    if ((rc = stream_alloc(st.get(), sizeof(__half) * n * L, &q))) { free_stream(st.get()); return rc; }
    st->h0 = static_cast<__half*>(q);
    if ((rc = stream_alloc(st.get(), sizeof(__half) * m_max * cmax, &q))) { free_stream(st.get()); return rc; }
    st->h = static_cast<__half*>(q);
    if ((rc = stream_alloc(st.get(), sizeof(float) * n * vxb_hop(c), &q))) { free_stream(st.get()); return rc; }
    st->out = static_cast<float*>(q);
    if ((rc = stream_zero(st.get(), c->stream))) { free_stream(st.get()); return rc; }
    for (int p = 0; p < 2; ++p) {
        Plan& P = st->set[p].plan;
        PlanSink sink(P);
        if ((rc = emit_stream_push(st.get(), p, sink))) { free_stream(st.get()); return rc; }
        CUDA_TRY(cudaStreamSynchronize(c->stream));
        CUDA_TRY(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        int orc = VXB_OK;
        for (auto& op : P.ops)
            if ((orc = op(c->stream))) break;
        cudaGraph_t graph = nullptr;
        const cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
        if (orc || e != cudaSuccess) {
            if (graph) cudaGraphDestroy(graph);
            free_stream(st.get());
            return orc ? orc : fail(VXB_ERR_BACKEND, std::string("stream graph capture: ") + cudaGetErrorString(e));
        }
        P.graph = graph;
        if (cudaGraphInstantiate(&P.exec, P.graph, 0) != cudaSuccess) {
            free_stream(st.get());
            return fail(VXB_ERR_BACKEND, "stream graph instantiate");
        }
    }
    if (cudaStreamSynchronize(c->stream) != cudaSuccess) {
        free_stream(st.get());
        return fail(VXB_ERR_BACKEND, "vxb_stream_open: device error");
    }
    *out = st.release();
    return VXB_OK;
}

extern "C" int vxb_stream_push_device(vxb_stream* st, const float* z_dev, float* out_dev, void* stream) {
    if (!st || !z_dev || !out_dev) return fail(VXB_ERR_INVALID_ARGUMENT, "null argument");
    vxb_ctx* c = st->c;
    DeviceGuard g(c->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    StreamSet& S = st->set[st->parity];
    const int n = st->n, L = c->latent_dim;
    // this push's frames into the latent window after its 6 history frames, channel by channel
    CUDA_TRY(cudaMemcpy2DAsync(S.z + 6, sizeof(float) * (6 + n), z_dev, sizeof(float) * n, sizeof(float) * n, L,
                               cudaMemcpyDeviceToDevice, s));
    CUDA_TRY(cudaMemsetAsync(c->status, 0, sizeof(int), s));
    CUDA_TRY(cudaGraphLaunch(S.plan.exec, s));
    CUDA_TRY(cudaMemcpyAsync(out_dev, st->out, sizeof(float) * n * vxb_hop(c), cudaMemcpyDeviceToDevice, s));
    CUDA_TRY(cudaMemcpyAsync(c->status_host, c->status, sizeof(int), cudaMemcpyDeviceToHost, s));
    st->parity ^= 1;
    return VXB_OK;
}

extern "C" int vxb_stream_push(vxb_stream* st, const float* z_host, float* out_host) {
    if (!st || !z_host || !out_host) return fail(VXB_ERR_INVALID_ARGUMENT, "null argument");
    vxb_ctx* c = st->c;
    DeviceGuard g(c->device);
    StreamSet& S = st->set[st->parity];
    const int n = st->n, L = c->latent_dim;
    CUDA_TRY(cudaMemcpy2DAsync(S.z + 6, sizeof(float) * (6 + n), z_host, sizeof(float) * n, sizeof(float) * n, L,
                               cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemsetAsync(c->status, 0, sizeof(int), c->stream));
    CUDA_TRY(cudaGraphLaunch(S.plan.exec, c->stream));
    CUDA_TRY(cudaMemcpyAsync(out_host, st->out, sizeof(float) * n * vxb_hop(c), cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaMemcpyAsync(c->status_host, c->status, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    st->parity ^= 1;
    int rc = wait_stream(c->stream, 60000);
    if (rc) return rc;
    return check_status(c);
}

extern "C" int vxb_stream_reset(vxb_stream* st) {
    if (!st) return fail(VXB_ERR_INVALID_ARGUMENT, "null stream");
    DeviceGuard g(st->c->device);
    CUDA_TRY(cudaStreamSynchronize(st->c->stream));
    int rc = stream_zero(st, st->c->stream);
    if (rc) return rc;
    CUDA_TRY(cudaStreamSynchronize(st->c->stream));
    return VXB_OK;
}

extern "C" int vxb_stream_close(vxb_stream* st) {
    if (!st) return VXB_OK;
    DeviceGuard g(st->c->device);
    cudaStreamSynchronize(st->c->stream);
    free_stream(st);
    delete st;
    return VXB_OK;
}
