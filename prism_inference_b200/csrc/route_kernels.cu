// route_kernels.cu - token routing for the grouped expert GEMM.
//
// The reference routes with an atomic per-expert count (moe_router.comp.glsl:50) and
// then dispatches every expert over every token, letting unrouted tokens return
// early (moe_expert_skip.comp.glsl:30; prism_moe_bench.cpp:428-436).  Its unused
// packed variant scatters tokens into per-expert buffers with atomics
// (moe_pack.comp.glsl:23-40).  Here the router's counts feed:
//   route_plan     one CTA: exclusive scan of the counts -> segment offsets, the list
//                  of 128-row tiles (expert, first sorted row, rows) and the tile
//                  count, then resets the counters for the next block;
//   route_scatter  every token takes a slot in its expert's segment, giving
//                  perm[sorted row] = token: ranks inside a 2048-token chunk from
//                  shared-memory atomics, one global atomic per (chunk, expert).
// The order of tokens inside a segment is not fixed, but each output row of the
// grouped GEMM depends only on its own input row, so results do not depend on it.
#include "common.cuh"
#include "route_kernels.cuh"
#include "tc_ffn.cuh"

namespace prism {

__global__ void __launch_bounds__(256) route_plan_kernel(RoutePlanArgs a) {
    __shared__ int s_off[256], s_toff[256];
    grid_dep_wait();  // the counts come from the attention kernel
    const int e = threadIdx.x;
    const int n = a.n_experts;
    const int c = e < n ? a.counts[e] : 0;
    s_off[e] = c;
    s_toff[e] = (c + 127) / 128;
    __syncthreads();
    // inclusive Hillis-Steele scans of counts and tile counts
    for (int d = 1; d < 256; d <<= 1) {
        const int v0 = e >= d ? s_off[e - d] : 0;
        const int v1 = e >= d ? s_toff[e - d] : 0;
        __syncthreads();
        s_off[e] += v0;
        s_toff[e] += v1;
        __syncthreads();
    }
    const int off = s_off[e] - c;                 // exclusive
    if (e < n) {
        a.offsets[e] = off;
        a.cursor[e] = 0;
        if (a.counts_out) a.counts_out[e] = c;
        a.counts[e] = 0;  // ready for the next block's router
    }
    // tile i belongs to the first expert whose inclusive tile count exceeds i; every
    // thread writes tiles i = tid, tid + 256, ... (coalesced records)
    const int n_tiles = s_toff[255];
    for (int i = e; i < n_tiles; i += 256) {
        int lo = 0, hi = 255;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (s_toff[mid] > i) hi = mid;
            else lo = mid + 1;
        }
        const int cnt = s_off[lo] - (lo > 0 ? s_off[lo - 1] : 0);
        const int j = i - (s_toff[lo] - (cnt + 127) / 128);  // tile index inside expert lo
        ExpertTile t;
        t.expert = lo;
        t.start = s_off[lo] - cnt + j * 128;
        t.rows = min(128, cnt - j * 128);
        t.pad = 0;
        a.tiles[i] = t;
    }
    if (e == 255) {
        *a.n_tiles = n_tiles;
        if (s_off[255] != a.n_tokens) atomicOr(a.err, ERR_ROUTE);  // every token routed exactly once
    }
}

// Tokens per scatter CTA: ranks inside an expert's share of the chunk come from shared
// atomics; one global atomic per (CTA, expert) reserves the share's rows.
constexpr int kScatterChunk = 2048;

__global__ void __launch_bounds__(256) route_scatter_kernel(RouteScatterArgs a) {
    __shared__ int s_cnt[256], s_base[256];
    constexpr int kPer = kScatterChunk / 256;
    const int t0 = blockIdx.x * kScatterChunk;
    s_cnt[threadIdx.x] = 0;
    grid_dep_wait();  // assignments (attention) and segment offsets (route_plan)
    __syncthreads();
    int ex[kPer], rk[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int t = t0 + i * 256 + threadIdx.x;
        int e = t < a.n_tokens ? a.assign[t] : -1;
        if (t < a.n_tokens && (e < 0 || e >= a.n_experts)) {
            atomicOr(a.err, ERR_ROUTE);
            e = -1;
        }
        ex[i] = e;
        rk[i] = e >= 0 ? atomicAdd(&s_cnt[e], 1) : 0;
    }
    __syncthreads();
    const int e = threadIdx.x;
    if (e < a.n_experts && s_cnt[e]) s_base[e] = a.offsets[e] + atomicAdd(&a.cursor[e], s_cnt[e]);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kPer; ++i)
        if (ex[i] >= 0) a.perm[s_base[ex[i]] + rk[i]] = t0 + i * 256 + threadIdx.x;
}

cudaError_t launch_route(const RoutePlanArgs& p, const RouteScatterArgs& s, cudaStream_t st) {
    cudaError_t e = launch_pdl(route_plan_kernel, dim3(1), dim3(256), 0, st, p);
    if (e != cudaSuccess) return e;
    if (s.n_tokens > 0)
        e = launch_pdl(route_scatter_kernel, dim3((s.n_tokens + kScatterChunk - 1) / kScatterChunk), dim3(256), 0, st,
                       s);
    return e;
}

}  // namespace prism
