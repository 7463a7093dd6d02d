// stack.cu - host side of libprism_moe.so: the C ABI of include/prism_moe.h.
//
// Replaces the reference's host dispatch (prism_moe_bench.cpp): instead of recording
// push constants + vkCmdDispatch + barrier per pass into a Vulkan command buffer, the
// entry points validate their arguments and launch stream-ordered CUDA kernels.
//  * per-pass drop-ins: one launch per reference dispatch (pass_kernels.cu)
//  * prism_stack_*: the whole stack over a batch of frames, with the weights repacked
//    once into aligned device arrays for TMA and the per-expert dispatch loop
//    replaced by route (route_kernels.cu) + one grouped tcgen05 GEMM (tc_ffn.cu).
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "attn_tc.cuh"
#include "common.cuh"
#include "host_util.h"
#include "pass_kernels.cuh"
#include "route_kernels.cuh"
#include "tc_ffn.cuh"

using namespace prism;

namespace {

thread_local std::string g_err;

}  // namespace

int prism::set_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

namespace {

#define fail prism::set_error

#define CUDA_TRY(x)                                                                          \
    do {                                                                                     \
        cudaError_t e_ = (x);                                                                \
        if (e_ != cudaSuccess) return fail(PRISM_E_CUDA, "%s: %s", #x, cudaGetErrorString(e_)); \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D fp16 row-major [rows][cols] tensor, box [box_rows][64] with 128-byte swizzle.
int make_map_2d(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return fail(PRISM_E_CUDA, "cuTensorMapEncodeTiled is not available");
    if (((uintptr_t)base & 15) || (cols * 2) % 16) return fail(PRISM_E_ALIGN, "tensor map base/stride not 16-byte aligned");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(PRISM_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return PRISM_OK;
}

// K-block-major fp16 weight [cols/64][rows][64] (see kb_major), box {64, box_rows, cols/64}:
// one load brings box_rows rows at their full K, one [box_rows][128 B] swizzled tile per
// 64-wide K-block.
int make_map_kb3d(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return fail(PRISM_E_CUDA, "cuTensorMapEncodeTiled is not available");
    if (((uintptr_t)base & 15) || cols % 64) return fail(PRISM_E_ALIGN, "K-block weight map: bad base or width");
    cuuint64_t dims[3] = {64, rows, cols / 64};
    cuuint64_t strides[2] = {128, rows * 128};
    cuuint32_t box[3] = {64, box_rows, (cuuint32_t)(cols / 64)};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(PRISM_E_CUDA, "cuTensorMapEncodeTiled (3d) failed (%d)", (int)r);
    return PRISM_OK;
}

// [rows][cols] -> [cols/64][rows][64]
std::vector<uint16_t> kb_major(const std::vector<uint16_t>& m, size_t rows, size_t cols) {
    std::vector<uint16_t> o(m.size());
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < cols; ++c) o[(c / 64) * rows * 64 + r * 64 + (c % 64)] = m[r * cols + c];
    return o;
}

// 4-D fp16 activation tensor (C, X=W, Y=H, F) HWC per frame, box {64, 8, 8, 1}, 128B swizzle:
// one box is one 8x8 window, 64 channels, rows in window-slot order.
int make_map_act4d(CUtensorMap* m, const void* base, int C, int W, int H, int F) {
    auto fn = encode_fn();
    if (!fn) return fail(PRISM_E_CUDA, "cuTensorMapEncodeTiled is not available");
    if ((uintptr_t)base & 15) return fail(PRISM_E_ALIGN, "activation buffer not 16-byte aligned");
    cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)F};
    cuuint64_t strides[3] = {(cuuint64_t)C * 2, (cuuint64_t)C * 2 * W, (cuuint64_t)C * 2 * W * H};
    cuuint32_t box[4] = {64, 8, 8, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(PRISM_E_CUDA, "cuTensorMapEncodeTiled (4d) failed (%d)", (int)r);
    return PRISM_OK;
}

float half_bits_to_float(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}

}  // namespace

// ============================== context =========================================

extern "C" int prism_abi_version(void) { return PRISM_ABI_VERSION; }
extern "C" const char* prism_last_error_string(void) { return g_err.c_str(); }

extern "C" int prism_create(int device, prism_ctx** out) {
    if (!out) return fail(PRISM_E_ARG, "prism_create: out is NULL");
    *out = nullptr;
    int n = 0;
    CUDA_TRY(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return fail(PRISM_E_ARG, "prism_create: device %d of %d", device, n);
    cudaDeviceProp prop;
    CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(PRISM_E_UNSUPPORTED, "prism_create: device %d is sm_%d%d; this library is built for sm_100a",
                    device, prop.major, prop.minor);
    DeviceGuard g(device);
    void* err = nullptr;
    if (cudaMalloc(&err, 4) != cudaSuccess || cudaMemset(err, 0, 4) != cudaSuccess) {
        cudaFree(err);
        return fail(PRISM_E_NOMEM, "prism_create: error word");
    }
    auto* c = new prism_ctx;
    c->device = device;
    c->sm_count = prop.multiProcessorCount;
    c->err = static_cast<uint32_t*>(err);
    c->codec = codec_scratch_new();
    *out = c;
    return PRISM_OK;
}

extern "C" int prism_destroy(prism_ctx* ctx) {
    if (!ctx) return PRISM_OK;
    {
        DeviceGuard g(ctx->device);
        cudaDeviceSynchronize();
        codec_scratch_free(ctx->codec);
        cudaFree(ctx->err);
    }
    delete ctx;
    return PRISM_OK;
}

// ============================== per-pass drop-ins ===============================

static int check_attn_shape(int dim, int n_heads, int head_dim, int ws, int W, int H, int n_tokens) {
    if (dim != 128 && dim != 256) return fail(PRISM_E_UNSUPPORTED, "dim %d (128 or 256)", dim);
    if (head_dim != 32 || n_heads * head_dim != dim)
        return fail(PRISM_E_UNSUPPORTED, "heads %d x %d for dim %d (head_dim 32)", n_heads, head_dim, dim);
    if (ws != 8) return fail(PRISM_E_UNSUPPORTED, "window_size %d (8)", ws);
    if (W <= 0 || H <= 0 || n_tokens <= 0) return fail(PRISM_E_ARG, "spatial %dx%d, n_tokens %d", W, H, n_tokens);
    return PRISM_OK;
}

extern "C" int prism_attn_window(prism_ctx* ctx, const prism_attn_params* p, const void* weights,
                                 size_t weight_elems, void* features, size_t feature_elems, void* stream) {
    if (!ctx || !p || !weights || !features) return fail(PRISM_E_ARG, "prism_attn_window: NULL argument");
    int rc = check_attn_shape(p->dim, p->n_heads, p->head_dim, p->window_size, p->spatial_w, p->spatial_h,
                              p->n_tokens);
    if (rc) return rc;
    const int64_t D = p->dim, T = (int64_t)p->spatial_w * p->spatial_h;
    if (!in_range(p->input_offset, T * D, feature_elems) || !in_range(p->output_offset, T * D, feature_elems))
        return fail(PRISM_E_RANGE, "prism_attn_window: feature offsets outside the arena");
    if (!in_range(p->qkv_w, 3 * D * D, weight_elems) || !in_range(p->qkv_b, 3 * D, weight_elems) ||
        !in_range(p->out_w, D * D, weight_elems) || !in_range(p->out_b, D, weight_elems))
        return fail(PRISM_E_RANGE, "prism_attn_window: weight offsets outside the blob");
    DeviceGuard g(ctx->device);
    AttnArgs a;
    a.weights = static_cast<const __half*>(weights);
    a.x = static_cast<const __half*>(features) + p->input_offset;
    a.y = static_cast<__half*>(features) + p->output_offset;
    a.frame_stride = T * D;
    a.qkv_w = p->qkv_w;
    a.qkv_b = p->qkv_b;
    a.out_w = p->out_w;
    a.out_b = p->out_b;
    a.W = p->spatial_w;
    a.H = p->spatial_h;
    a.n_tokens = p->n_tokens;
    a.scale = 0.1767766953f;  // 1/sqrt(32), split2_qkv_attn_d256.comp.glsl:62
    CUDA_TRY(launch_attn_window(a, p->dim, 1, as_stream(stream)));
    return PRISM_OK;
}

extern "C" int prism_router(prism_ctx* ctx, const prism_router_params* p, const void* weights,
                            size_t weight_elems, const void* features, size_t feature_elems, int32_t* aux,
                            size_t aux_elems, void* stream) {
    if (!ctx || !p || !weights || !features || !aux) return fail(PRISM_E_ARG, "prism_router: NULL argument");
    if (p->dim != 128 && p->dim != 256) return fail(PRISM_E_UNSUPPORTED, "prism_router: dim %d", p->dim);
    if (p->n_experts < 1 || p->n_experts > 256)
        return fail(PRISM_E_UNSUPPORTED, "prism_router: n_experts %d (1..256)", p->n_experts);
    if (p->n_tokens < 0) return fail(PRISM_E_ARG, "prism_router: n_tokens %d", p->n_tokens);
    const int64_t D = p->dim, T = p->n_tokens, N = p->n_experts;
    if (!in_range(p->input_offset, T * D, feature_elems))
        return fail(PRISM_E_RANGE, "prism_router: input outside the arena");
    if (!in_range(p->assignment_offset, T, aux_elems) || !in_range(p->count_offset, N, aux_elems))
        return fail(PRISM_E_RANGE, "prism_router: aux offsets outside the aux arena");
    if (!in_range(p->router_w, N * D, weight_elems) || !in_range(p->router_b, N, weight_elems))
        return fail(PRISM_E_RANGE, "prism_router: weight offsets outside the blob");
    DeviceGuard g(ctx->device);
    RouterArgs a;
    a.weights = static_cast<const __half*>(weights);
    a.x = static_cast<const __half*>(features) + p->input_offset;
    a.assign = aux + p->assignment_offset;
    a.counts = aux + p->count_offset;
    a.router_w = p->router_w;
    a.router_b = p->router_b;
    a.n_experts = p->n_experts;
    a.n_tokens = p->n_tokens;
    CUDA_TRY(launch_router(a, p->dim, as_stream(stream)));
    return PRISM_OK;
}

extern "C" int prism_expert(prism_ctx* ctx, const prism_expert_params* p, const void* weights,
                            size_t weight_elems, void* features, size_t feature_elems, const int32_t* aux,
                            size_t aux_elems, void* stream) {
    if (!ctx || !p || !weights || !features || !aux) return fail(PRISM_E_ARG, "prism_expert: NULL argument");
    if (p->dim != 128 && p->dim != 256) return fail(PRISM_E_UNSUPPORTED, "prism_expert: dim %d", p->dim);
    if (p->n_tokens < 0) return fail(PRISM_E_ARG, "prism_expert: n_tokens %d", p->n_tokens);
    const int64_t D = p->dim, T = p->n_tokens;
    if (!in_range(p->input_offset, T * D, feature_elems) || !in_range(p->output_offset, T * D, feature_elems))
        return fail(PRISM_E_RANGE, "prism_expert: feature offsets outside the arena");
    if (!in_range(p->assignment_offset, T, aux_elems))
        return fail(PRISM_E_RANGE, "prism_expert: assignment outside the aux arena");
    if (!in_range(p->w1_offset, D * D, weight_elems) || !in_range(p->b1_offset, D, weight_elems) ||
        !in_range(p->w2_offset, D * D, weight_elems) || !in_range(p->b2_offset, D, weight_elems))
        return fail(PRISM_E_RANGE, "prism_expert: weight offsets outside the blob");
    DeviceGuard g(ctx->device);
    ExpertArgs a;
    a.weights = static_cast<const __half*>(weights);
    a.x = static_cast<const __half*>(features) + p->input_offset;
    a.y = static_cast<__half*>(features) + p->output_offset;
    a.assign = aux + p->assignment_offset;
    a.w1 = p->w1_offset;
    a.b1 = p->b1_offset;
    a.w2 = p->w2_offset;
    a.b2 = p->b2_offset;
    a.expert_id = p->expert_id;
    a.n_tokens = p->n_tokens;
    CUDA_TRY(launch_expert(a, p->dim, as_stream(stream)));
    return PRISM_OK;
}

static int proj_common(prism_ctx* ctx, const prism_proj_params* p, const void* weights, size_t weight_elems,
                       void* features, size_t feature_elems, void* stream, bool up) {
    const char* name = up ? "prism_proj_up" : "prism_proj_down";
    if (!ctx || !p || !weights || !features) return fail(PRISM_E_ARG, "%s: NULL argument", name);
    if (p->n_tokens < 0) return fail(PRISM_E_ARG, "%s: n_tokens %d", name, p->n_tokens);
    const int64_t T = p->n_tokens, K = up ? 128 : 256, N = up ? 256 : 128;
    if (!in_range(p->input_offset, T * K, feature_elems) || !in_range(p->output_offset, T * N, feature_elems))
        return fail(PRISM_E_RANGE, "%s: feature offsets outside the arena", name);
    if (!in_range(p->w_offset, N * K, weight_elems) || !in_range(p->b_offset, N, weight_elems))
        return fail(PRISM_E_RANGE, "%s: weight offsets outside the blob", name);
    DeviceGuard g(ctx->device);
    ProjArgs a;
    a.weights = static_cast<const __half*>(weights);
    a.x = static_cast<const __half*>(features) + p->input_offset;
    a.y = static_cast<__half*>(features) + p->output_offset;
    a.w = p->w_offset;
    a.b = p->b_offset;
    a.n_tokens = p->n_tokens;
    CUDA_TRY(launch_proj(a, up, as_stream(stream)));
    return PRISM_OK;
}

extern "C" int prism_proj_up(prism_ctx* ctx, const prism_proj_params* p, const void* weights, size_t weight_elems,
                             void* features, size_t feature_elems, void* stream) {
    return proj_common(ctx, p, weights, weight_elems, features, feature_elems, stream, true);
}
extern "C" int prism_proj_down(prism_ctx* ctx, const prism_proj_params* p, const void* weights,
                               size_t weight_elems, void* features, size_t feature_elems, void* stream) {
    return proj_common(ctx, p, weights, weight_elems, features, feature_elems, stream, false);
}

extern "C" int prism_dense_block(prism_ctx* ctx, const prism_dense_params* p, int32_t ffn_hidden,
                                 int32_t ffn_chunk, const void* weights, size_t weight_elems, void* features,
                                 size_t feature_elems, void* stream) {
    if (!ctx || !p || !weights || !features) return fail(PRISM_E_ARG, "prism_dense_block: NULL argument");
    int rc = check_attn_shape(p->dim, p->n_heads, p->head_dim, p->window_size, p->spatial_w, p->spatial_h,
                              p->n_tokens);
    if (rc) return rc;
    if (ffn_hidden <= 0 || ffn_chunk <= 0 || ffn_hidden % ffn_chunk || ffn_chunk > 512 || ffn_chunk % 32)
        return fail(PRISM_E_UNSUPPORTED, "prism_dense_block: ffn_hidden %d / ffn_chunk %d", ffn_hidden, ffn_chunk);
    const int64_t D = p->dim, T = (int64_t)p->spatial_w * p->spatial_h, Hd = ffn_hidden;
    if (!in_range(p->input_offset, T * D, feature_elems) || !in_range(p->output_offset, T * D, feature_elems))
        return fail(PRISM_E_RANGE, "prism_dense_block: feature offsets outside the arena");
    if (!in_range(p->qkv_w_offset, 3 * D * D, weight_elems) || !in_range(p->qkv_b_offset, 3 * D, weight_elems) ||
        !in_range(p->out_w_offset, D * D, weight_elems) || !in_range(p->out_b_offset, D, weight_elems) ||
        !in_range(p->ffn_w1_offset, Hd * D, weight_elems) || !in_range(p->ffn_b1_offset, Hd, weight_elems) ||
        !in_range(p->ffn_w2_offset, D * Hd, weight_elems) || !in_range(p->ffn_b2_offset, D, weight_elems))
        return fail(PRISM_E_RANGE, "prism_dense_block: weight offsets outside the blob");
    DeviceGuard g(ctx->device);
    AttnArgs a;
    a.weights = static_cast<const __half*>(weights);
    a.x = static_cast<const __half*>(features) + p->input_offset;
    a.y = static_cast<__half*>(features) + p->output_offset;
    a.frame_stride = T * D;
    a.qkv_w = p->qkv_w_offset;
    a.qkv_b = p->qkv_b_offset;
    a.out_w = p->out_w_offset;
    a.out_b = p->out_b_offset;
    a.W = p->spatial_w;
    a.H = p->spatial_h;
    a.n_tokens = p->n_tokens;
    a.scale = 0.1767766953f;
    CUDA_TRY(launch_attn_window(a, p->dim, 1, as_stream(stream)));
    DenseFfnArgs f;
    f.weights = a.weights;
    f.io = a.y;
    f.w1 = p->ffn_w1_offset;
    f.b1 = p->ffn_b1_offset;
    f.w2 = p->ffn_w2_offset;
    f.b2 = p->ffn_b2_offset;
    f.hidden = ffn_hidden;
    f.chunk = ffn_chunk;
    f.n_tokens = (int)T;
    CUDA_TRY(launch_dense_ffn(f, p->dim, as_stream(stream)));
    return PRISM_OK;
}

// ============================== fast path ======================================

namespace {

// Bucket routing needs max_experts * rows int32 slots (a bucket per expert that could take every
// token); above this budget the route kernel builds a compact permutation instead.
constexpr size_t kBucketBudget = 256ull << 20;

struct FastBlock {
    prism_block_desc d;
    __half* w1 = nullptr;  // experts: [E][256][256]; dense: [hidden][D]
    __half* w2 = nullptr;  // experts: [E][256][256]; dense: [D][hidden]
    float* b1 = nullptr;   // [E][256] / [hidden]
    float* b2 = nullptr;   // [E][256] / [D]
    CUtensorMap tm_w1, tm_w2;
    int moe_index = -1;
    // fused attention: head-major QKV, out-projection, padded router (MoE blocks, D = 256)
    __half* wqkv = nullptr;  // [3D][D], rows of head h at 96h: q(32) k(32) v(32)
    float* bqkv = nullptr;   // [3D] same order
    __half* wo = nullptr;    // [D][D]
    float* bo = nullptr;     // [D]
    __half* wr = nullptr;    // [npad][256], rows >= n_experts zero
    float* br = nullptr;     // [npad]
    int npad = 0;
    CUtensorMap tm_wqkv, tm_wo, tm_wr;
};

}  // namespace

struct prism_stack {
    prism_ctx* ctx = nullptr;
    prism_stack_desc desc;
    std::vector<prism_block_desc> bdesc;
    int T = 0, max_frames = 0, n_moe = 0;
    __half* blob = nullptr;
    size_t blob_elems = 0;
    __half *up_w = nullptr, *dn_w = nullptr;
    float *up_b = nullptr, *dn_b = nullptr;
    CUtensorMap tm_up, tm_dn, tm_act_a, tm_act_b, tm_act_y;
    std::vector<FastBlock> blocks;
    __half *act_a = nullptr, *act_b = nullptr, *act_y = nullptr;
    int32_t *assign_ws = nullptr, *counts = nullptr, *cursor = nullptr, *perm = nullptr,
            *n_tiles = nullptr;
    // bucket routing (PRISM_OPT_BUCKET_ROUTING): the router writes each expert's tokens into a
    // bucket of `rows` slots and the expert kernel plans its tiles from the counts, so no route
    // kernel runs; allocated when max_experts * rows int32 fit kBucketBudget
    int32_t* perm_b = nullptr;
    uint32_t* route_done = nullptr;
    bool bucket_routing = false;   // buffers allocated
    bool use_buckets = true;        // PRISM_OPT_BUCKET_ROUTING
    ExpertTile* tiles = nullptr;
    uint32_t* err = nullptr;
    std::vector<void*> allocs;
    // host-buffer inference (prism_stack_infer / _submit / _wait): two device staging slots,
    // an upload and a download stream, created on first use
    struct Staging {
        bool ready = false;
        __half *in[2] = {}, *out[2] = {};
        cudaStream_t s_in = nullptr, s_out = nullptr, s_fwd = nullptr;
        cudaEvent_t in_ready[2] = {}, out_done[2] = {}, t0[2] = {}, t1[2] = {};
        int64_t next = 0;  // ticket of the next submission; slot = ticket & 1
    } stg;
    // PRISM_OPT_PAIR_ATTENTION: dim-256 attention of forwards with at most sm_count / 2 tiles
    // runs with each tile's heads split over a CTA pair (attn_pair.cu)
    bool pair_attention = true;
    int max_experts = 0;
    // per-kernel profiling (prism_stack_profile)
    bool profiling = false;
    std::vector<cudaEvent_t> ev_pool;
    size_t ev_used = 0;
    std::vector<int> ev_kind;  // kind of each recorded (start, end) pair
};

namespace {

template <typename T>
int dev_alloc(prism_stack* st, T** p, size_t count) {
    void* q = nullptr;
    if (cudaMalloc(&q, count * sizeof(T) + 16) != cudaSuccess)
        return fail(PRISM_E_NOMEM, "cudaMalloc of %zu bytes failed", count * sizeof(T));
    st->allocs.push_back(q);
    *p = static_cast<T*>(q);
    return PRISM_OK;
}

void free_staging(prism_stack* st) {
    auto& q = st->stg;
    for (int i = 0; i < 2; ++i) {
        for (cudaEvent_t* e : {&q.in_ready[i], &q.out_done[i], &q.t0[i], &q.t1[i]})
            if (*e) cudaEventDestroy(*e), *e = nullptr;
        if (q.in[i]) cudaFree(q.in[i]), q.in[i] = nullptr;
        if (q.out[i]) cudaFree(q.out[i]), q.out[i] = nullptr;
    }
    for (cudaStream_t* s : {&q.s_in, &q.s_out, &q.s_fwd})
        if (*s) cudaStreamDestroy(*s), *s = nullptr;
    q.ready = false;
}

void free_stack(prism_stack* st) {
    free_staging(st);
    for (void* p : st->allocs) cudaFree(p);
    st->allocs.clear();
    for (cudaEvent_t e : st->ev_pool) cudaEventDestroy(e);
    st->ev_pool.clear();
}

// Brackets one launch with events when profiling is on.
struct KernelTimer {
    prism_stack* st;
    cudaStream_t s;
    int kind;
    cudaEvent_t end = nullptr;
    KernelTimer(prism_stack* st_, cudaStream_t s_, int kind_) : st(st_), s(s_), kind(kind_) {
        if (!st->profiling) return;
        while (st->ev_pool.size() < st->ev_used + 2) {
            cudaEvent_t e;
            if (cudaEventCreate(&e) != cudaSuccess) return;
            st->ev_pool.push_back(e);
        }
        cudaEventRecord(st->ev_pool[st->ev_used], s);
        end = st->ev_pool[st->ev_used + 1];
        st->ev_used += 2;
        st->ev_kind.push_back(kind);
    }
    ~KernelTimer() {
        if (end) cudaEventRecord(end, s);
    }
};

int validate_desc(const prism_stack_desc* d, size_t elems) {
    int rc = check_attn_shape(d->dim, d->n_heads, d->head_dim, d->window_size, d->spatial_w, d->spatial_h, 1);
    if (rc) return rc;
    const int64_t D = d->dim;
    if (d->n_blocks < 0 || (d->n_blocks > 0 && !d->blocks)) return fail(PRISM_E_ARG, "n_blocks %d", d->n_blocks);
    if (d->up_w >= 0) {
        if (D != 256 || d->in_dim != 128) return fail(PRISM_E_UNSUPPORTED, "up adapter needs dim 256, in_dim 128");
        if (!in_range(d->up_w, 256 * 128, elems) || !in_range(d->up_b, 256, elems))
            return fail(PRISM_E_RANGE, "up adapter outside the blob");
    } else if (d->in_dim != D) {
        return fail(PRISM_E_ARG, "in_dim %d without adapter", d->in_dim);
    }
    if (d->down_w >= 0) {
        if (D != 256 || d->out_dim != 128) return fail(PRISM_E_UNSUPPORTED, "down adapter needs dim 256, out_dim 128");
        if (!in_range(d->down_w, 128 * 256, elems) || !in_range(d->down_b, 128, elems))
            return fail(PRISM_E_RANGE, "down adapter outside the blob");
    } else if (d->out_dim != D) {
        return fail(PRISM_E_ARG, "out_dim %d without adapter", d->out_dim);
    }
    for (int i = 0; i < d->n_blocks; ++i) {
        const prism_block_desc& b = d->blocks[i];
        if (!in_range(b.qkv_w, 3 * D * D, elems) || !in_range(b.qkv_b, 3 * D, elems) ||
            !in_range(b.out_w, D * D, elems) || !in_range(b.out_b, D, elems))
            return fail(PRISM_E_RANGE, "block %d: attention weights outside the blob", i);
        if (b.kind == PRISM_BLOCK_MOE) {
            if (D != 256) return fail(PRISM_E_UNSUPPORTED, "block %d: MoE blocks need dim 256", i);
            if (b.n_experts < 1 || b.n_experts > 256) return fail(PRISM_E_UNSUPPORTED, "block %d: n_experts %d", i, b.n_experts);
            if (!in_range(b.router_w, b.n_experts * D, elems) || !in_range(b.router_b, b.n_experts, elems))
                return fail(PRISM_E_RANGE, "block %d: router outside the blob", i);
            const int64_t last = (int64_t)(b.n_experts - 1) * b.expert_stride;
            if (b.expert_stride < 0 || !in_range(b.expert_w1, last + D * D, elems) ||
                !in_range(b.expert_b1, last + D, elems) || !in_range(b.expert_w2, last + D * D, elems) ||
                !in_range(b.expert_b2, last + D, elems))
                return fail(PRISM_E_RANGE, "block %d: experts outside the blob", i);
        } else if (b.kind == PRISM_BLOCK_DENSE) {
            const int64_t Hd = b.ffn_hidden;
            if (Hd <= 0 || b.ffn_chunk <= 0 || Hd % b.ffn_chunk || b.ffn_chunk > 512 || b.ffn_chunk % 32)
                return fail(PRISM_E_UNSUPPORTED, "block %d: ffn_hidden %d / ffn_chunk %d", i, b.ffn_hidden, b.ffn_chunk);
            if (D == 256 && b.ffn_chunk != 256)
                return fail(PRISM_E_UNSUPPORTED, "block %d: dim-256 dense FFN needs ffn_chunk 256", i);
            if (D == 128 && ffn_dense128_w1_box(b.ffn_hidden, b.ffn_chunk) == 0)
                return fail(PRISM_E_UNSUPPORTED,
                            "block %d: dim-128 dense FFN %d / chunk %d (chunk == hidden: 128 or a multiple of 256; "
                            "or chunk 128 / 256 dividing hidden)",
                            i, b.ffn_hidden, b.ffn_chunk);
            if (!in_range(b.ffn_w1, Hd * D, elems) || !in_range(b.ffn_b1, Hd, elems) ||
                !in_range(b.ffn_w2, D * Hd, elems) || !in_range(b.ffn_b2, D, elems))
                return fail(PRISM_E_RANGE, "block %d: FFN weights outside the blob", i);
        } else {
            return fail(PRISM_E_ARG, "block %d: kind %d", i, b.kind);
        }
    }
    return PRISM_OK;
}

template <typename T>
int upload(prism_stack* st, T** dst, const std::vector<T>& src) {
    int rc = dev_alloc(st, dst, src.size());
    if (rc) return rc;
    CUDA_TRY(cudaMemcpy(*dst, src.data(), src.size() * sizeof(T), cudaMemcpyHostToDevice));
    return PRISM_OK;
}

}  // namespace

extern "C" int prism_stack_create(prism_ctx* ctx, const prism_stack_desc* desc, const void* blob, size_t blob_elems,
                                  int blob_on_host, int max_frames, prism_stack** out) {
    if (!ctx || !desc || !blob || !out) return fail(PRISM_E_ARG, "prism_stack_create: NULL argument");
    *out = nullptr;
    if (max_frames < 1) return fail(PRISM_E_ARG, "prism_stack_create: max_frames %d", max_frames);
    int rc = validate_desc(desc, blob_elems);
    if (rc) return rc;
    DeviceGuard g(ctx->device);
    if (!blob_on_host) {
        cudaPointerAttributes attr;
        if (cudaPointerGetAttributes(&attr, blob) != cudaSuccess || attr.type != cudaMemoryTypeDevice ||
            attr.device != ctx->device)
            return fail(PRISM_E_ARG, "prism_stack_create: blob is not device memory of device %d", ctx->device);
    }
    const int64_t T = (int64_t)desc->spatial_w * desc->spatial_h;
    const int64_t rows = T * max_frames;
    if (rows > (int64_t)1 << 30) return fail(PRISM_E_RANGE, "prism_stack_create: %lld tokens", (long long)rows);

    auto* st = new prism_stack;
    st->ctx = ctx;
    st->desc = *desc;
    st->bdesc.assign(desc->blocks, desc->blocks + desc->n_blocks);
    st->desc.blocks = st->bdesc.data();
    st->T = (int)T;
    st->max_frames = max_frames;

    // host copy of the blob (repacking is done on the host once)
    std::vector<uint16_t> hb;
    const uint16_t* hblob = static_cast<const uint16_t*>(blob);
    if (!blob_on_host) {
        hb.resize(blob_elems);
        if (cudaMemcpy(hb.data(), blob, blob_elems * 2, cudaMemcpyDeviceToHost) != cudaSuccess) {
            delete st;
            return fail(PRISM_E_CUDA, "prism_stack_create: blob download failed");
        }
        hblob = hb.data();
    }
    auto fail_cleanup = [&](int code) {
        free_stack(st);
        delete st;
        return code;
    };
    // raw blob on the device (the attention / router kernels address it by element offset)
    if ((rc = dev_alloc(st, &st->blob, blob_elems))) return fail_cleanup(rc);
    st->blob_elems = blob_elems;
    if (cudaMemcpy(st->blob, hblob, blob_elems * 2, cudaMemcpyHostToDevice) != cudaSuccess)
        return fail_cleanup(fail(PRISM_E_CUDA, "blob upload failed"));

    auto copy_mat = [&](std::vector<uint16_t>& dst, size_t dst_off, int64_t src_off, int64_t rows_, int64_t cols,
                        int64_t src_ld) {
        for (int64_t r = 0; r < rows_; ++r)
            memcpy(&dst[dst_off + r * cols], hblob + src_off + r * src_ld, cols * 2);
    };
    auto copy_bias = [&](std::vector<float>& dst, size_t dst_off, int64_t src_off, int64_t n) {
        for (int64_t i = 0; i < n; ++i) dst[dst_off + i] = half_bits_to_float(hblob[src_off + i]);
    };
    if (desc->up_w >= 0) {
        std::vector<uint16_t> w(256 * 128);
        std::vector<float> b(256);
        copy_mat(w, 0, desc->up_w, 256, 128, 128);
        copy_bias(b, 0, desc->up_b, 256);
        if ((rc = upload(st, (uint16_t**)&st->up_w, w)) || (rc = upload(st, &st->up_b, b))) return fail_cleanup(rc);
        if ((rc = make_map_2d(&st->tm_up, st->up_w, 256, 128, 256))) return fail_cleanup(rc);
    }
    if (desc->down_w >= 0) {
        std::vector<uint16_t> w(128 * 256);
        std::vector<float> b(128);
        copy_mat(w, 0, desc->down_w, 128, 256, 256);
        copy_bias(b, 0, desc->down_b, 128);
        if ((rc = upload(st, (uint16_t**)&st->dn_w, w)) || (rc = upload(st, &st->dn_b, b))) return fail_cleanup(rc);
        if ((rc = make_map_2d(&st->tm_dn, st->dn_w, 128, 256, 128))) return fail_cleanup(rc);
    }
    const int64_t D = desc->dim;
    int max_experts = 1;
    for (int i = 0; i < desc->n_blocks; ++i) {
        FastBlock fb;
        fb.d = desc->blocks[i];
        {
            // head-major Wqkv: the q, k and v rows of head h (32 each) at rows 96h .. 96h + 95
            const int heads = (int)(D / 32);
            std::vector<uint16_t> wqkv((size_t)3 * D * D), wo((size_t)D * D);
            std::vector<float> bqkv(3 * D), bo(D);
            for (int h = 0; h < heads; ++h)
                for (int part = 0; part < 3; ++part) {
                    copy_mat(wqkv, (size_t)(h * 96 + part * 32) * D, fb.d.qkv_w + (int64_t)(part * D + h * 32) * D, 32,
                             D, D);
                    copy_bias(bqkv, h * 96 + part * 32, fb.d.qkv_b + part * D + h * 32, 32);
                }
            copy_mat(wo, 0, fb.d.out_w, D, D, D);
            copy_bias(bo, 0, fb.d.out_b, D);
            // Wqkv K-block-major: one TMA load brings a head's 96 rows at full K
            if ((rc = upload(st, (uint16_t**)&fb.wqkv, kb_major(wqkv, 3 * D, D))) || (rc = upload(st, &fb.bqkv, bqkv)) ||
                (rc = upload(st, (uint16_t**)&fb.wo, wo)) || (rc = upload(st, &fb.bo, bo)))
                return fail_cleanup(rc);
            if ((rc = make_map_kb3d(&fb.tm_wqkv, fb.wqkv, 3 * D, D, 96)) || (rc = make_map_2d(&fb.tm_wo, fb.wo, D, D, D)))
                return fail_cleanup(rc);
            if (fb.d.kind == PRISM_BLOCK_MOE) {
                fb.npad = (fb.d.n_experts + 15) / 16 * 16;
                std::vector<uint16_t> wr((size_t)fb.npad * 256, 0);
                std::vector<float> br(fb.npad, 0.0f);
                copy_mat(wr, 0, fb.d.router_w, fb.d.n_experts, 256, 256);
                copy_bias(br, 0, fb.d.router_b, fb.d.n_experts);
                if ((rc = upload(st, (uint16_t**)&fb.wr, kb_major(wr, fb.npad, 256))) || (rc = upload(st, &fb.br, br)))
                    return fail_cleanup(rc);
                if ((rc = make_map_kb3d(&fb.tm_wr, fb.wr, fb.npad, 256, std::min(96, fb.npad)))) return fail_cleanup(rc);
            } else {
                fb.tm_wr = fb.tm_wo;  // unused without a router
            }
        }
        if (fb.d.kind == PRISM_BLOCK_MOE) {
            fb.moe_index = st->n_moe++;
            const int E = fb.d.n_experts;
            max_experts = std::max(max_experts, E);
            std::vector<uint16_t> w1((size_t)E * D * D), w2((size_t)E * D * D);
            std::vector<float> b1((size_t)E * D), b2((size_t)E * D);
            for (int e = 0; e < E; ++e) {
                const int64_t eo = (int64_t)e * fb.d.expert_stride;
                copy_mat(w1, (size_t)e * D * D, fb.d.expert_w1 + eo, D, D, D);
                copy_mat(w2, (size_t)e * D * D, fb.d.expert_w2 + eo, D, D, D);
                copy_bias(b1, (size_t)e * D, fb.d.expert_b1 + eo, D);
                copy_bias(b2, (size_t)e * D, fb.d.expert_b2 + eo, D);
            }
            if ((rc = upload(st, (uint16_t**)&fb.w1, w1)) || (rc = upload(st, (uint16_t**)&fb.w2, w2)) ||
                (rc = upload(st, &fb.b1, b1)) || (rc = upload(st, &fb.b2, b2)))
                return fail_cleanup(rc);
            if ((rc = make_map_2d(&fb.tm_w1, fb.w1, (uint64_t)E * D, D, 256)) ||
                (rc = make_map_2d(&fb.tm_w2, fb.w2, (uint64_t)E * D, D, 256)))
                return fail_cleanup(rc);
        } else {
            const int64_t Hd = fb.d.ffn_hidden;
            std::vector<uint16_t> w1((size_t)Hd * D), w2((size_t)D * Hd);
            std::vector<float> b1(Hd), b2(D);
            copy_mat(w1, 0, fb.d.ffn_w1, Hd, D, D);
            copy_mat(w2, 0, fb.d.ffn_w2, D, Hd, Hd);
            copy_bias(b1, 0, fb.d.ffn_b1, Hd);
            copy_bias(b2, 0, fb.d.ffn_b2, D);
            if ((rc = upload(st, (uint16_t**)&fb.w1, w1)) || (rc = upload(st, (uint16_t**)&fb.w2, w2)) ||
                (rc = upload(st, &fb.b1, b1)) || (rc = upload(st, &fb.b2, b2)))
                return fail_cleanup(rc);
            // W1 K-chunks of one GEMM1 piece (256 rows at D = 256; 128 or 256 at D = 128), W2 of
            // all D output rows
            const uint32_t w1_box = D == 256 ? 256u : (uint32_t)ffn_dense128_w1_box((int)Hd, fb.d.ffn_chunk);
            if ((rc = make_map_2d(&fb.tm_w1, fb.w1, Hd, D, w1_box)) || (rc = make_map_2d(&fb.tm_w2, fb.w2, D, Hd, (uint32_t)D)))
                return fail_cleanup(rc);
        }
        st->blocks.push_back(fb);
    }
    // workspace
    if ((rc = dev_alloc(st, &st->act_a, rows * D)) || (rc = dev_alloc(st, &st->act_b, rows * D)) ||
        (rc = dev_alloc(st, &st->act_y, rows * D)) || (rc = dev_alloc(st, &st->assign_ws, rows)) ||
        (rc = dev_alloc(st, &st->counts, 256)) ||
        (rc = dev_alloc(st, &st->cursor, 256)) || (rc = dev_alloc(st, &st->perm, rows)) ||
        (rc = dev_alloc(st, &st->n_tiles, 1)) || (rc = dev_alloc(st, &st->tiles, rows / 128 + 256 + 1)) ||
        (rc = dev_alloc(st, &st->err, 1)))
        return fail_cleanup(rc);
    if (cudaMemset(st->counts, 0, 256 * 4) != cudaSuccess || cudaMemset(st->cursor, 0, 256 * 4) != cudaSuccess ||
        cudaMemset(st->err, 0, 4) != cudaSuccess)
        return fail_cleanup(fail(PRISM_E_CUDA, "workspace memset failed"));
    st->max_experts = st->n_moe ? max_experts : 0;
    if (st->n_moe && (size_t)max_experts * rows * 4 <= kBucketBudget) {
        if ((rc = dev_alloc(st, &st->perm_b, (size_t)max_experts * rows)) || (rc = dev_alloc(st, &st->route_done, 1)))
            return fail_cleanup(rc);
        if (cudaMemset(st->route_done, 0, 4) != cudaSuccess)
            return fail_cleanup(fail(PRISM_E_CUDA, "workspace memset failed"));
        st->bucket_routing = true;
    }
    {
        if ((rc = make_map_2d(&st->tm_act_a, st->act_a, rows, D, 128)) ||
            (rc = make_map_2d(&st->tm_act_b, st->act_b, rows, D, 128)) ||
            (rc = make_map_2d(&st->tm_act_y, st->act_y, rows, D, 128)))
            return fail_cleanup(rc);
    }
    if (cudaDeviceSynchronize() != cudaSuccess) return fail_cleanup(fail(PRISM_E_CUDA, "stack upload failed"));
    *out = st;
    return PRISM_OK;
}

extern "C" int prism_stack_destroy(prism_stack* st) {
    if (!st) return PRISM_OK;
    DeviceGuard g(st->ctx->device);
    cudaDeviceSynchronize();
    free_stack(st);
    delete st;
    return PRISM_OK;
}

extern "C" int prism_stack_tokens_per_frame(const prism_stack* st) { return st ? st->T : 0; }

extern "C" int prism_stack_launch_count(const prism_stack* st, int frames) {
    if (!st || frames <= 0) return 0;
    int n = (st->desc.up_w >= 0 ? 1 : 0) + (st->desc.down_w >= 0 ? 1 : 0);
    // MoE (dim 256): attention with the fused router, routing, experts; dense: attention, FFN
    const bool buckets = st->bucket_routing && st->use_buckets;
    for (const auto& b : st->blocks) n += b.d.kind == PRISM_BLOCK_MOE && !buckets ? 3 : 2;
    if (st->desc.down_w < 0 && st->blocks.empty()) n += 1;  // plain copy
    return n;
}

extern "C" int prism_stack_status(prism_stack* st, void* stream) {
    if (!st) return fail(PRISM_E_ARG, "prism_stack_status: NULL");
    DeviceGuard g(st->ctx->device);
    uint32_t e = 0;
    CUDA_TRY(cudaMemcpyAsync(&e, st->err, 4, cudaMemcpyDeviceToHost, as_stream(stream)));
    CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
    CUDA_TRY(cudaMemsetAsync(st->err, 0, 4, as_stream(stream)));
    if (e) {  // a forward that gave up may have left routing counts behind: start the next one clean
        CUDA_TRY(cudaMemsetAsync(st->counts, 0, 256 * 4, as_stream(stream)));
        CUDA_TRY(cudaMemsetAsync(st->cursor, 0, 256 * 4, as_stream(stream)));
        if (st->route_done) CUDA_TRY(cudaMemsetAsync(st->route_done, 0, 4, as_stream(stream)));
    }
    CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
    if (e & ERR_TIMEOUT) return fail(PRISM_E_TIMEOUT, "a device-side wait timed out (error word 0x%x)", e);
    if (e & ERR_ROUTE) return fail(PRISM_E_RANGE, "routing invariant failed (error word 0x%x)", e);
    return PRISM_OK;
}

// Diagnostic stall: one warp adds a token to expert 0's routing count, as a router cut short
// in mid-block leaves it, then waits through the library's bounded mbarrier wait on a barrier
// that nothing arrives at.  The wait gives up after kWaitLimitNs and the kernel records
// ERR_TIMEOUT in the stack's error word, as a stack kernel whose wait ran out does.
__global__ void __launch_bounds__(32) stall_kernel(int32_t* counts, uint32_t* err) {
    __shared__ uint64_t bar;
    __shared__ int gave_up;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        gave_up = 0;
        fence_barrier_init();
        atomicAdd(&counts[0], 1);
    }
    __syncwarp();
    if (!mbar_wait_w(&bar, 0, &gave_up) && threadIdx.x == 0) atomicOr(err, ERR_TIMEOUT);
}

extern "C" int prism_stack_inject_stall(prism_stack* st, void* stream) {
    if (!st) return fail(PRISM_E_ARG, "prism_stack_inject_stall: NULL");
    DeviceGuard g(st->ctx->device);
    stall_kernel<<<1, 32, 0, as_stream(stream)>>>(st->counts, st->err);
    CUDA_TRY(cudaGetLastError());
    return PRISM_OK;
}

namespace {

// The whole stack; counts_out (nullable, one-MoE-block stacks) receives the block's per-expert
// token counts as the routing kernel reads them.
int stack_forward(prism_stack* st, const void* in, void* out, int frames, int32_t* assign, int32_t* counts_out,
                  void* stream) {
    if (!st) return fail(PRISM_E_ARG, "prism_stack_forward: NULL stack");
    if (frames < 0 || frames > st->max_frames)
        return fail(PRISM_E_RANGE, "prism_stack_forward: frames %d (max %d)", frames, st->max_frames);
    if (frames == 0) return PRISM_OK;  // an empty batch: nothing to read or write
    if (!in || !out) return fail(PRISM_E_ARG, "prism_stack_forward: NULL argument");
    if (in == out) return fail(PRISM_E_ARG, "prism_stack_forward: out aliases in");
    DeviceGuard g(st->ctx->device);
    cudaStream_t s = as_stream(stream);
    const prism_stack_desc& d = st->desc;
    const int D = d.dim, T = st->T;
    const int rows = T * frames;
    const int grid = st->ctx->sm_count;
    int rc;

    const __half* cur = static_cast<const __half*>(in);
    const CUtensorMap* cur_map = nullptr;
    CUtensorMap tm_in;
    if (d.up_w >= 0) {
        if ((rc = make_map_2d(&tm_in, in, rows, 128, 128))) return rc;
        FfnArgs a{};
        a.x = static_cast<const __half*>(in);
        a.y = st->act_a;
        a.n_rows = rows;
        a.b1 = st->up_b;
        a.err = st->err;
        KernelTimer kt(st, s, PRISM_K_PROJ_UP);
        CUDA_TRY(launch_ffn_proj_up(a, tm_in, st->tm_up, std::min(grid, (rows + 127) / 128), s));
        cur = st->act_a;
        cur_map = &st->tm_act_a;
    }
    const int nb = (int)st->blocks.size();
    for (int bi = 0; bi < nb; ++bi) {
        const FastBlock& b = st->blocks[bi];
        const bool last = bi == nb - 1;
        // output of this block: the caller's buffer if nothing follows, else a ping-pong buffer
        __half* nxt;
        const CUtensorMap* nxt_map;
        if (last && d.down_w < 0) {
            nxt = static_cast<__half*>(out);
            nxt_map = nullptr;
        } else if (cur == st->act_a) {
            nxt = st->act_b;
            nxt_map = &st->tm_act_b;
        } else {
            nxt = st->act_a;
            nxt_map = &st->tm_act_a;
        }
        // fused tcgen05 attention (+ router, histogram): x (cur) -> y (act_y)
        int32_t* asg = assign ? assign + (size_t)std::max(b.moe_index, 0) * rows : st->assign_ws;
        CUtensorMap tm_x, tm_y;
        if ((rc = make_map_act4d(&tm_x, cur, D, d.spatial_w, d.spatial_h, frames)) ||
            (rc = make_map_act4d(&tm_y, st->act_y, D, d.spatial_w, d.spatial_h, frames)))
            return rc;
        AttnTcArgs ta;
        ta.W = d.spatial_w;
        ta.H = d.spatial_h;
        ta.frames = frames;
        ta.n_keys = std::min(64, T);
        ta.n_experts = b.d.kind == PRISM_BLOCK_MOE ? b.d.n_experts : 0;
        ta.n_experts_pad = b.npad;
        ta.scale = 0.1767766953f;
        ta.bqkv = b.bqkv;
        ta.bo = b.bo;
        ta.br = b.br;
        ta.assign = asg;
        ta.counts = st->counts;
        const bool buckets = b.d.kind == PRISM_BLOCK_MOE && st->bucket_routing && st->use_buckets;
        ta.perm_b = buckets ? st->perm_b : nullptr;
        ta.perm_stride = (int)rows;
        ta.err = st->err;
        const int n_win = ((d.spatial_w + 7) / 8) * ((d.spatial_h + 7) / 8) * frames;
        {
            KernelTimer kt(st, s, PRISM_K_ATTN);
            const int n_attn_tiles = (n_win + 1) / 2;
            if (D == 256 && st->pair_attention && 2 * n_attn_tiles <= grid)
                CUDA_TRY(launch_attn_pair(ta, tm_x, tm_y, b.tm_wqkv, b.tm_wo, b.tm_wr, n_attn_tiles, s));
            else
                CUDA_TRY(launch_attn_tc(D, ta, tm_x, tm_y, b.tm_wqkv, b.tm_wo, b.tm_wr, std::min(grid, n_attn_tiles), s));
        }
        if (b.d.kind == PRISM_BLOCK_MOE && buckets) {
            // the router filled the buckets: the expert kernel plans its tiles from the counts
            FfnArgs fa{};
            fa.x = st->act_y;
            fa.y = nxt;
            fa.perm = st->perm_b;
            fa.tiles = nullptr;
            fa.n_tiles = nullptr;
            fa.perm_stride = (int)rows;
            fa.route_done = st->route_done;
            fa.counts_out = counts_out;
            fa.b1 = b.b1;
            fa.b2 = b.b2;
            fa.err = st->err;
            fa.route_counts = st->counts;
            fa.route_cursor = nullptr;
            fa.n_route = b.d.n_experts;
            fa.n_rows = (int)rows;
            KernelTimer kt(st, s, PRISM_K_EXPERT);
            CUDA_TRY(launch_ffn_expert256(fa, b.tm_w1, b.tm_w2, grid, s));
        } else if (b.d.kind == PRISM_BLOCK_MOE) {
            RouteArgs ra_;
            ra_.counts = st->counts;
            ra_.counts_out = counts_out;
            ra_.cursor = st->cursor;
            ra_.assign = asg;
            ra_.perm = st->perm;
            ra_.tiles = st->tiles;
            ra_.n_tiles = st->n_tiles;
            ra_.n_experts = b.d.n_experts;
            ra_.n_tokens = rows;
            ra_.err = st->err;
            {
                KernelTimer kt(st, s, PRISM_K_ROUTE);
                CUDA_TRY(launch_route(ra_, s));
            }
            FfnArgs fa{};
            fa.x = st->act_y;
            fa.y = nxt;
            fa.perm = st->perm;
            fa.tiles = st->tiles;
            fa.n_tiles = st->n_tiles;
            fa.b1 = b.b1;
            fa.b2 = b.b2;
            fa.err = st->err;
            fa.route_counts = st->counts;
            fa.route_cursor = st->cursor;
            fa.n_route = b.d.n_experts;
            KernelTimer kt(st, s, PRISM_K_EXPERT);
            fa.n_rows = (int)rows;
            CUDA_TRY(launch_ffn_expert256(fa, b.tm_w1, b.tm_w2,
                                          std::min(grid, rows / 128 + b.d.n_experts), s));
        } else {
            FfnArgs fa{};
            fa.x = st->act_y;
            fa.y = nxt;
            fa.n_rows = rows;
            fa.b1 = b.b1;
            fa.b2 = b.b2;
            fa.err = st->err;
            KernelTimer kt(st, s, PRISM_K_DENSE_FFN);
            if (D == 256)
                CUDA_TRY(launch_ffn_dense256(fa, st->tm_act_y, b.tm_w1, b.tm_w2, b.d.ffn_hidden / 256,
                                             std::min(grid, (rows + 127) / 128), s));
            else
                CUDA_TRY(launch_ffn_dense128(fa, st->tm_act_y, b.tm_w1, b.tm_w2, b.d.ffn_hidden, b.d.ffn_chunk,
                                             std::min(grid, (rows + 127) / 128), s));
        }
        cur = nxt;
        cur_map = nxt_map;
    }
    if (d.down_w >= 0) {
        const CUtensorMap* xm = cur_map;
        CUtensorMap tm_cur;
        if (!xm) {  // no blocks and no up adapter: x is the caller's input
            if ((rc = make_map_2d(&tm_cur, cur, rows, 256, 128))) return rc;
            xm = &tm_cur;
        }
        FfnArgs a{};
        a.x = cur;
        a.y = static_cast<__half*>(out);
        a.n_rows = rows;
        a.b1 = st->dn_b;
        a.err = st->err;
        KernelTimer kt(st, s, PRISM_K_PROJ_DOWN);
        CUDA_TRY(launch_ffn_proj_down(a, *xm, st->tm_dn, std::min(grid, (rows + 127) / 128), s));
    } else if (nb == 0) {
        KernelTimer kt(st, s, PRISM_K_COPY);
        CUDA_TRY(cudaMemcpyAsync(out, cur, (size_t)rows * D * 2, cudaMemcpyDeviceToDevice, s));
    }
    return PRISM_OK;
}

}  // namespace

extern "C" int prism_stack_forward(prism_stack* st, const void* in, void* out, int frames, int32_t* assign,
                                   void* stream) {
    return stack_forward(st, in, out, frames, assign, nullptr, stream);
}

extern "C" int prism_moe_block(prism_stack* blk, const void* features_in, void* features_out, int frames,
                               int32_t* assign, int32_t* counts, void* stream) {
    if (!blk) return fail(PRISM_E_ARG, "prism_moe_block: NULL block");
    if (blk->desc.n_blocks != 1 || blk->desc.blocks[0].kind != PRISM_BLOCK_MOE || blk->desc.up_w >= 0 ||
        blk->desc.down_w >= 0)
        return fail(PRISM_E_ARG, "prism_moe_block: the handle must hold exactly one MoE block and no adapters");
    return stack_forward(blk, features_in, features_out, frames, assign, counts, stream);
}

// ---- host-buffer inference -------------------------------------------------------------
// The reference's Infer uploads the frame through a staging buffer, runs the recorded
// command buffer, waits on a fence and downloads the result (prism_vulkan.cpp:1007-1040).
// Here two device staging slots let one submission's upload and the previous one's download
// run on their own streams while the forward in between computes: per slot, the upload waits
// for the forward that last read the slot, the forward waits for the upload and for the
// download that last read its output slot, and the download waits for the forward.

namespace {

int staging_init(prism_stack* st) {
    auto& q = st->stg;
    if (q.ready) return PRISM_OK;
    const size_t rows = (size_t)st->T * st->max_frames;
    bool ok = true;
    for (int i = 0; i < 2 && ok; ++i) {
        ok = cudaMalloc(&q.in[i], rows * st->desc.in_dim * 2) == cudaSuccess &&
             cudaMalloc(&q.out[i], rows * st->desc.out_dim * 2) == cudaSuccess &&
             cudaEventCreateWithFlags(&q.in_ready[i], cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreateWithFlags(&q.out_done[i], cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreate(&q.t0[i]) == cudaSuccess && cudaEventCreate(&q.t1[i]) == cudaSuccess;
    }
    for (cudaStream_t* s : {&q.s_in, &q.s_out, &q.s_fwd})
        ok = ok && cudaStreamCreateWithFlags(s, cudaStreamNonBlocking) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        free_staging(st);
        return fail(PRISM_E_NOMEM, "host-buffer staging: allocation of 2 x %zu frames' buffers failed",
                    (size_t)st->max_frames);
    }
    q.ready = true;
    return PRISM_OK;
}

}  // namespace

extern "C" int prism_stack_submit(prism_stack* st, const void* host_in, void* host_out, int frames, void* stream,
                                  int64_t* ticket) {
    if (!st) return fail(PRISM_E_ARG, "prism_stack_submit: NULL stack");
    if (frames < 0 || frames > st->max_frames)
        return fail(PRISM_E_RANGE, "prism_stack_submit: frames %d (max %d)", frames, st->max_frames);
    if (frames > 0 && !host_in) return fail(PRISM_E_ARG, "prism_stack_submit: NULL host_in");
    DeviceGuard g(st->ctx->device);
    int rc = staging_init(st);
    if (rc) return rc;
    auto& q = st->stg;
    const int64_t k = q.next;
    const int p = (int)(k & 1);
    cudaStream_t s = as_stream(stream);
    const size_t rows = (size_t)st->T * frames;
    const size_t in_bytes = rows * st->desc.in_dim * 2, out_bytes = rows * st->desc.out_dim * 2;
    // upload, once the forward that last read this slot is done (t1 of the slot)
    CUDA_TRY(cudaStreamWaitEvent(q.s_in, q.t1[p], 0));
    if (in_bytes) CUDA_TRY(cudaMemcpyAsync(q.in[p], host_in, in_bytes, cudaMemcpyHostToDevice, q.s_in));
    CUDA_TRY(cudaEventRecord(q.in_ready[p], q.s_in));
    // forward, once the upload has landed and the slot's previous output has been downloaded
    CUDA_TRY(cudaStreamWaitEvent(s, q.in_ready[p], 0));
    CUDA_TRY(cudaStreamWaitEvent(s, q.out_done[p], 0));
    CUDA_TRY(cudaEventRecord(q.t0[p], s));
    if ((rc = prism_stack_forward(st, q.in[p], q.out[p], frames, nullptr, stream))) return rc;
    CUDA_TRY(cudaEventRecord(q.t1[p], s));
    // download
    if (host_out && out_bytes) {
        CUDA_TRY(cudaStreamWaitEvent(q.s_out, q.t1[p], 0));
        CUDA_TRY(cudaMemcpyAsync(host_out, q.out[p], out_bytes, cudaMemcpyDeviceToHost, q.s_out));
        CUDA_TRY(cudaEventRecord(q.out_done[p], q.s_out));
    } else {
        CUDA_TRY(cudaEventRecord(q.out_done[p], s));
    }
    q.next = k + 1;
    if (ticket) *ticket = k;
    return PRISM_OK;
}

extern "C" int prism_stack_wait(prism_stack* st, int64_t ticket, void* stream) {
    if (!st) return fail(PRISM_E_ARG, "prism_stack_wait: NULL stack");
    if (ticket < 0 || ticket >= st->stg.next)
        return fail(PRISM_E_RANGE, "prism_stack_wait: ticket %lld was not submitted", (long long)ticket);
    DeviceGuard g(st->ctx->device);
    // a later submission to the same slot completes after this one, so its event covers it
    cudaEvent_t e = st->stg.out_done[ticket & 1];
    if (stream) CUDA_TRY(cudaStreamWaitEvent(as_stream(stream), e, 0));
    else CUDA_TRY(cudaEventSynchronize(e));
    return PRISM_OK;
}

extern "C" int prism_stack_infer_gpu(prism_stack* st, const void* in_buf, size_t in_offset, void* out_buf,
                                     size_t out_offset, int frames, float* gpu_ms) {
    if (!st) return fail(PRISM_E_ARG, "prism_stack_infer_gpu: NULL stack");
    if (frames < 0 || frames > st->max_frames)
        return fail(PRISM_E_RANGE, "prism_stack_infer_gpu: frames %d (max %d)", frames, st->max_frames);
    if (gpu_ms) *gpu_ms = 0.0f;
    if (frames == 0) return PRISM_OK;
    if (!in_buf || !out_buf) return fail(PRISM_E_ARG, "prism_stack_infer_gpu: NULL buffer");
    DeviceGuard g(st->ctx->device);
    for (const void* p : {in_buf, (const void*)out_buf}) {
        cudaPointerAttributes attr;
        if (cudaPointerGetAttributes(&attr, p) != cudaSuccess || attr.type != cudaMemoryTypeDevice ||
            attr.device != st->ctx->device) {
            cudaGetLastError();
            return fail(PRISM_E_ARG, "prism_stack_infer_gpu: buffers must be device memory of device %d",
                        st->ctx->device);
        }
    }
    const size_t rows = (size_t)st->T * frames;
    const size_t in_bytes = rows * st->desc.in_dim * 2, out_bytes = rows * st->desc.out_dim * 2;
    const char* in = static_cast<const char*>(in_buf) + in_offset;
    char* out = static_cast<char*>(out_buf) + out_offset;
    if (in < out + out_bytes && out < in + in_bytes)
        return fail(PRISM_E_ARG, "prism_stack_infer_gpu: the output range overlaps the input range");
    int rc = staging_init(st);  // the internal stream and timing events (and, if needed, the slots)
    if (rc) return rc;
    auto& q = st->stg;
    cudaStream_t s = q.s_fwd;
    // the slot's events of the host-buffer path order this call after any earlier submission
    const int p = (int)(q.next & 1);
    CUDA_TRY(cudaStreamWaitEvent(s, q.out_done[p], 0));
    const bool direct = ((uintptr_t)in & 15) == 0 && ((uintptr_t)out & 15) == 0;
    if (!direct) CUDA_TRY(cudaMemcpyAsync(q.in[p], in, in_bytes, cudaMemcpyDeviceToDevice, s));
    CUDA_TRY(cudaEventRecord(q.t0[p], s));
    if ((rc = prism_stack_forward(st, direct ? in : (const char*)q.in[p], direct ? out : (char*)q.out[p], frames,
                                  nullptr, s)))
        return rc;
    CUDA_TRY(cudaEventRecord(q.t1[p], s));
    if (!direct) CUDA_TRY(cudaMemcpyAsync(out, q.out[p], out_bytes, cudaMemcpyDeviceToDevice, s));
    CUDA_TRY(cudaEventRecord(q.out_done[p], s));
    q.next += 1;
    CUDA_TRY(cudaEventSynchronize(q.out_done[p]));
    if (gpu_ms) CUDA_TRY(cudaEventElapsedTime(gpu_ms, q.t0[p], q.t1[p]));
    return prism_stack_status(st, s);
}

extern "C" int prism_stack_infer(prism_stack* st, const void* host_in, void* host_out, int frames, float* gpu_ms) {
    if (!st) return fail(PRISM_E_ARG, "prism_stack_infer: NULL stack");
    DeviceGuard g(st->ctx->device);
    int rc = staging_init(st);
    if (rc) return rc;
    int64_t k = 0;
    if ((rc = prism_stack_submit(st, host_in, host_out, frames, st->stg.s_fwd, &k))) return rc;
    const int p = (int)(k & 1);
    CUDA_TRY(cudaEventSynchronize(st->stg.out_done[p]));
    if (gpu_ms) CUDA_TRY(cudaEventElapsedTime(gpu_ms, st->stg.t0[p], st->stg.t1[p]));
    return prism_stack_status(st, st->stg.s_fwd);
}

extern "C" int prism_stack_set_option(prism_stack* st, int option, int value) {
    if (!st) return fail(PRISM_E_ARG, "prism_stack_set_option: NULL");
    switch (option) {
        case PRISM_OPT_PAIR_ATTENTION:
            st->pair_attention = value != 0;
            return PRISM_OK;
        case PRISM_OPT_BUCKET_ROUTING:
            st->use_buckets = value != 0;
            return PRISM_OK;
        default:
            return fail(PRISM_E_ARG, "prism_stack_set_option: unknown option %d", option);
    }
}

extern "C" int prism_stack_profile(prism_stack* st, int enable) {
    if (!st) return fail(PRISM_E_ARG, "prism_stack_profile: NULL");
    st->profiling = enable != 0;
    return PRISM_OK;
}

extern "C" int prism_stack_profile_read(prism_stack* st, double* ms, int64_t* launches, int n_kinds) {
    if (!st || !ms || !launches || n_kinds < 0) return fail(PRISM_E_ARG, "prism_stack_profile_read: NULL");
    DeviceGuard g(st->ctx->device);
    for (int k = 0; k < n_kinds; ++k) {
        ms[k] = 0.0;
        launches[k] = 0;
    }
    if (st->ev_used) CUDA_TRY(cudaEventSynchronize(st->ev_pool[st->ev_used - 1]));
    for (size_t i = 0; i < st->ev_kind.size(); ++i) {
        float t = 0.0f;
        CUDA_TRY(cudaEventElapsedTime(&t, st->ev_pool[2 * i], st->ev_pool[2 * i + 1]));
        const int k = st->ev_kind[i];
        if (k < n_kinds) {
            ms[k] += t;
            launches[k] += 1;
        }
    }
    st->ev_used = 0;
    st->ev_kind.clear();
    return PRISM_OK;
}
