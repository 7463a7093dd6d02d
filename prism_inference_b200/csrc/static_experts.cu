// static_experts.cu - prism_expert_all_static: all experts of one MoE pass in one
// call, with no device allocation at all.
//
// Who needs it.  Prism is meant to run as a post-process inside someone else's frame
// loop (a game or driver hook that is handed device buffers it did not create).  Such
// a caller cannot call cudaMalloc when the pass runs: allocation can synchronize the
// device and stall the host application's frame, and many hosts allow device
// allocation only at start-up, if at all.  The regular grouped path needs scratch
// (per-expert counts, offsets, the token permutation and the tile list) that
// prism_stack_create allocates; this entry point keeps that scratch in a file-scope
// device array instead, so the caller passes only inputs and outputs.
//
// What it computes: the same as calling prism_expert once per expert
// (moe_expert_skip.comp.glsl:25-54 dispatched N times, prism_moe_bench.cpp:428-436),
// but the tokens are grouped by expert first (counts -> offsets -> permutation) and
// one launch processes 32-token tiles of every expert, on the CUDA cores with the
// reference's order of operations (cta_mv.cuh).
//
// The scratch array g_expert_scratch (PRISM_STATIC_MAX_TOKENS tokens, about 300 KB)
// exists on every GPU that loads the library, for as long as the process runs.
#include <mutex>

#include "common.cuh"
#include "cta_mv.cuh"
#include "host_util.h"

namespace {

constexpr int kMaxTokens = PRISM_STATIC_MAX_TOKENS;
constexpr int kMaxExperts = 256;
constexpr int kTileRows = 32;
constexpr int kMaxTiles = kMaxTokens / kTileRows + kMaxExperts;
// layout of the scratch array, in int32 words
constexpr int kOffCounts = 0;      // [256] tokens per expert
constexpr int kOffOffsets = 256;   // [256] first sorted row of each expert
constexpr int kOffCursor = 512;    // [256] scatter cursors
constexpr int kOffNTiles = 768;    // [1]   number of tiles
constexpr int kOffTiles = 1024;    // [kMaxTiles][4] (expert, first sorted row, rows, -)
constexpr int kOffPerm = kOffTiles + 4 * kMaxTiles;  // [kMaxTokens] sorted row -> token
constexpr int kScratchWords = kOffPerm + kMaxTokens;

}  // namespace

static __device__ __align__(256) int32_t g_expert_scratch[kScratchWords];

namespace prism {
namespace {

struct StaticExpertArgs {
    int32_t* scratch;        // device address of g_expert_scratch on this device
    const __half* weights;
    const __half* x;         // input rows (features + input_offset)
    __half* y;               // output rows (features + output_offset)
    const int32_t* assign;   // aux + assignment_offset
    int w1, b1, w2, b2, stride;
    int first_expert, n_experts, n_tokens;
};

// The counters must start at zero on every call: the previous call left its counts.
__global__ void se_reset(StaticExpertArgs a) {
    for (int e = threadIdx.x; e < kMaxExperts; e += blockDim.x) {
        a.scratch[kOffCounts + e] = 0;
        a.scratch[kOffCursor + e] = 0;
    }
}

// expert (relative to first_expert) of token t, or -1 when no expert of this call owns it
__device__ __forceinline__ int rel_expert(const StaticExpertArgs& a, int t) {
    const int e = a.assign[t] - a.first_expert;
    return (e >= 0 && e < a.n_experts) ? e : -1;
}

__global__ void se_count(StaticExpertArgs a) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    const int e = t < a.n_tokens ? rel_expert(a, t) : -1;
    const unsigned peers = __match_any_sync(__activemask(), e);
    if (e >= 0 && (int)(threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&a.scratch[kOffCounts + e], __popc(peers));
}

__global__ void se_plan(StaticExpertArgs a) {
    __shared__ int s_off[kMaxExperts], s_toff[kMaxExperts];
    const int e = threadIdx.x;
    const int c = e < a.n_experts ? a.scratch[kOffCounts + e] : 0;
    s_off[e] = c;
    s_toff[e] = (c + kTileRows - 1) / kTileRows;
    __syncthreads();
    for (int d = 1; d < kMaxExperts; d <<= 1) {
        const int v0 = e >= d ? s_off[e - d] : 0, v1 = e >= d ? s_toff[e - d] : 0;
        __syncthreads();
        s_off[e] += v0;
        s_toff[e] += v1;
        __syncthreads();
    }
    const int nt = (c + kTileRows - 1) / kTileRows;
    const int off = s_off[e] - c, toff = s_toff[e] - nt;
    if (e < a.n_experts) {
        a.scratch[kOffOffsets + e] = off;
        for (int j = 0; j < nt; ++j) {
            int32_t* t = a.scratch + kOffTiles + 4 * (toff + j);
            t[0] = e;
            t[1] = off + j * kTileRows;
            t[2] = min(kTileRows, c - j * kTileRows);
        }
    }
    if (e == kMaxExperts - 1) a.scratch[kOffNTiles] = s_toff[e];
}

__global__ void se_scatter(StaticExpertArgs a) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    const int e = t < a.n_tokens ? rel_expert(a, t) : -1;
    const unsigned lanes = __activemask();
    const unsigned peers = __match_any_sync(lanes, e);
    const int leader = __ffs(peers) - 1;
    int base = 0;
    if (e >= 0 && (int)(threadIdx.x & 31) == leader) base = atomicAdd(&a.scratch[kOffCursor + e], __popc(peers));
    base = __shfl_sync(lanes, base, leader);
    if (e >= 0)
        a.scratch[kOffPerm + a.scratch[kOffOffsets + e] + base + __popc(peers & ((1u << (threadIdx.x & 31)) - 1))] = t;
}

// One CTA per tile of up to 32 tokens of one expert:
// z = h( MV(W2, b2, gelu_h(MV(W1, b1, y))) + y )   (moe_expert_skip.comp.glsl:32-53)
template <int D>
__global__ void __launch_bounds__(256) se_expert(StaticExpertArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    float* Xs = reinterpret_cast<float*>(smem);  // [32][D]
    float* Hs = Xs + kTileRows * D;              // [32][D]
    float* Rs = Hs + kTileRows * D;              // [32][D]
    __shared__ int tok[kTileRows];
    if ((int)blockIdx.x >= a.scratch[kOffNTiles]) return;
    const int32_t* tile = a.scratch + kOffTiles + 4 * blockIdx.x;
    const int e = tile[0], start = tile[1], rows = tile[2];
    if (threadIdx.x < kTileRows) tok[threadIdx.x] = threadIdx.x < rows ? a.scratch[kOffPerm + start + threadIdx.x] : 0;
    __syncthreads();
    for (int i = threadIdx.x; i < kTileRows * D; i += blockDim.x) {
        const int t = i / D;
        Xs[i] = t < rows ? __half2float(a.x[(size_t)tok[t] * D + (i % D)]) : 0.0f;
    }
    __syncthreads();
    const int64_t eo = (int64_t)e * a.stride;
    cta_mv<kTileRows>(a.weights + a.w1 + eo, D, a.weights + a.b1 + eo, D, D, Xs, D, Hs, D);
    __syncthreads();
    for (int i = threadIdx.x; i < kTileRows * D; i += blockDim.x) Hs[i] = rh(gelu_exact(Hs[i]));
    __syncthreads();
    cta_mv<kTileRows>(a.weights + a.w2 + eo, D, a.weights + a.b2 + eo, D, D, Hs, D, Rs, D);
    __syncthreads();
    for (int i = threadIdx.x; i < rows * D; i += blockDim.x) {
        const int t = i / D, c = i % D;
        a.y[(size_t)tok[t] * D + c] = __float2half_rn(__fadd_rn(Rs[i], Xs[i]));
    }
}

// Device address of g_expert_scratch, looked up once per device with that device
// current (host code cannot use the symbol itself as a device pointer).
std::mutex g_scratch_mu;
int32_t* g_scratch_ptr[128] = {};

int32_t* scratch_on(int device) {
    if (device < 0 || device >= 128) return nullptr;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[device]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_expert_scratch) != cudaSuccess) return nullptr;
        g_scratch_ptr[device] = static_cast<int32_t*>(p);
    }
    return g_scratch_ptr[device];
}

}  // namespace
}  // namespace prism

using namespace prism;

extern "C" int prism_expert_all_static(prism_ctx* ctx, const prism_expert_params* p, int32_t n_experts,
                                       int32_t expert_stride, const void* weights, size_t weight_elems,
                                       void* features, size_t feature_elems, const int32_t* aux, size_t aux_elems,
                                       void* stream) {
    if (!ctx || !p || !weights || !features || !aux)
        return set_error(PRISM_E_ARG, "prism_expert_all_static: NULL argument");
    if (p->dim != 128 && p->dim != 256) return set_error(PRISM_E_UNSUPPORTED, "prism_expert_all_static: dim %d", p->dim);
    if (p->n_tokens < 0 || p->n_tokens > kMaxTokens)
        return set_error(PRISM_E_RANGE,
                         "prism_expert_all_static: n_tokens %d exceeds the static scratch limit of %d tokens "
                         "(PRISM_STATIC_MAX_TOKENS); use the allocating prism_stack_* path for larger passes",
                         p->n_tokens, kMaxTokens);
    if (n_experts < 1 || n_experts > kMaxExperts)
        return set_error(PRISM_E_UNSUPPORTED, "prism_expert_all_static: n_experts %d (1..%d)", n_experts, kMaxExperts);
    if (expert_stride < 0) return set_error(PRISM_E_ARG, "prism_expert_all_static: expert_stride %d", expert_stride);
    const int64_t D = p->dim, T = p->n_tokens, last = (int64_t)(n_experts - 1) * expert_stride;
    if (!in_range(p->input_offset, T * D, feature_elems) || !in_range(p->output_offset, T * D, feature_elems))
        return set_error(PRISM_E_RANGE, "prism_expert_all_static: feature offsets outside the arena");
    if (!in_range(p->assignment_offset, T, aux_elems))
        return set_error(PRISM_E_RANGE, "prism_expert_all_static: assignment outside the aux arena");
    if (!in_range(p->w1_offset, last + D * D, weight_elems) || !in_range(p->b1_offset, last + D, weight_elems) ||
        !in_range(p->w2_offset, last + D * D, weight_elems) || !in_range(p->b2_offset, last + D, weight_elems))
        return set_error(PRISM_E_RANGE, "prism_expert_all_static: expert weights outside the blob");
    if (T == 0) return PRISM_OK;
    DeviceGuard g(ctx->device);
    int32_t* scratch = scratch_on(ctx->device);
    if (!scratch) return set_error(PRISM_E_CUDA, "prism_expert_all_static: cudaGetSymbolAddress failed");
    StaticExpertArgs a;
    a.scratch = scratch;
    a.weights = static_cast<const __half*>(weights);
    a.x = static_cast<const __half*>(features) + p->input_offset;
    a.y = static_cast<__half*>(features) + p->output_offset;
    a.assign = aux + p->assignment_offset;
    a.w1 = p->w1_offset;
    a.b1 = p->b1_offset;
    a.w2 = p->w2_offset;
    a.b2 = p->b2_offset;
    a.stride = expert_stride;
    a.first_expert = p->expert_id;
    a.n_experts = n_experts;
    a.n_tokens = (int)T;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int blocks = (int)((T + 255) / 256);
    se_reset<<<1, 256, 0, s>>>(a);
    se_count<<<blocks, 256, 0, s>>>(a);
    se_plan<<<1, kMaxExperts, 0, s>>>(a);
    se_scatter<<<blocks, 256, 0, s>>>(a);
    const int max_tiles = (int)((T + kTileRows - 1) / kTileRows) + n_experts;
    const size_t smem = (size_t)3 * kTileRows * D * 4;
    cudaError_t e;
    if (D == 256) {
        e = cudaFuncSetAttribute(se_expert<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) se_expert<256><<<max_tiles, 256, smem, s>>>(a);
    } else {
        e = cudaFuncSetAttribute(se_expert<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) se_expert<128><<<max_tiles, 256, smem, s>>>(a);
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(PRISM_E_CUDA, "prism_expert_all_static: %s", cudaGetErrorString(e));
    return PRISM_OK;
}
