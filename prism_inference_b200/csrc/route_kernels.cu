// route_kernels.cu - token routing for the grouped expert GEMM.
//
// The reference routes with an atomic per-expert count (moe_router.comp.glsl:50) and
// then dispatches every expert over every token, letting unrouted tokens return
// early (moe_expert_skip.comp.glsl:30; prism_moe_bench.cpp:428-436).  Its unused
// packed variant scatters tokens into per-expert buffers with atomics
// (moe_pack.comp.glsl:23-40).  Here one kernel turns the router's counts into:
//   - segment offsets: every CTA scans the (at most 256) counts itself, so no separate
//     planning launch is needed;
//   - the list of 128-row tiles (expert, first sorted row, rows) and the tile count,
//     written by CTA 0;
//   - perm[sorted row] = token: each CTA takes a 2048-token chunk, ranks inside the chunk
//     from shared-memory atomics, one global atomic per (chunk, expert) on the cursors.
// The counts and cursors are cleared by the expert kernel that follows (it runs after this
// kernel and before the next block's router adds to them).
// The order of tokens inside a segment is not fixed, but each output row of the
// grouped GEMM depends only on its own input row, so results do not depend on it.
#include "common.cuh"
#include "route_kernels.cuh"
#include "tc_ffn.cuh"

namespace prism {

// Tokens per CTA: ranks inside an expert's share of the chunk come from shared atomics;
// one global atomic per (CTA, expert) reserves the share's rows.
constexpr int kScatterChunk = 2048;

__global__ void __launch_bounds__(256) route_kernel(RouteArgs a) {
    __shared__ int s_off[256], s_toff[256], s_cnt[256], s_base[256];
    const int e = threadIdx.x;
    const int n = a.n_experts;
    s_cnt[e] = 0;
    grid_dep_wait();  // counts and assignments come from the router
    grid_dep_launch();  // short kernel: the expert kernel may launch (it waits for this one)
    // inclusive Hillis-Steele scans of the counts and of the tile counts
    const int c = e < n ? a.counts[e] : 0;
    s_off[e] = c;
    s_toff[e] = (c + 127) / 128;
    __syncthreads();
    for (int d = 1; d < 256; d <<= 1) {
        const int v0 = e >= d ? s_off[e - d] : 0;
        const int v1 = e >= d ? s_toff[e - d] : 0;
        __syncthreads();
        s_off[e] += v0;
        s_toff[e] += v1;
        __syncthreads();
    }
    // Counts that do not add up to the token count (left behind by a forward that gave up)
    // would place rows outside the permutation and tile arrays: flag it, plan no tiles and
    // scatter nothing.  The expert kernel that follows then has no work and clears the counts.
    if (s_off[255] != a.n_tokens) {
        if (blockIdx.x == 0 && e == 0) {
            *a.n_tiles = 0;
            atomicOr(a.err, ERR_ROUTE);
        }
        return;
    }
    if (blockIdx.x == 0) {
        if (e < n && a.counts_out) a.counts_out[e] = c;
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
        if (e == 255) *a.n_tiles = n_tiles;
    }
    // ---- this CTA's chunk of tokens
    constexpr int kPer = kScatterChunk / 256;
    const int t0 = blockIdx.x * kScatterChunk;
    int ex[kPer], rk[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int t = t0 + i * 256 + threadIdx.x;
        int ee = t < a.n_tokens ? a.assign[t] : -1;
        if (t < a.n_tokens && (ee < 0 || ee >= n)) {
            atomicOr(a.err, ERR_ROUTE);
            ee = -1;
        }
        ex[i] = ee;
        rk[i] = ee >= 0 ? atomicAdd(&s_cnt[ee], 1) : 0;
    }
    __syncthreads();
    if (e < n && s_cnt[e]) s_base[e] = (s_off[e] - c) + atomicAdd(&a.cursor[e], s_cnt[e]);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kPer; ++i)
        if (ex[i] >= 0) a.perm[s_base[ex[i]] + rk[i]] = t0 + i * 256 + threadIdx.x;
}

cudaError_t launch_route(const RouteArgs& a, cudaStream_t st) {
    const int grid = a.n_tokens > 0 ? (a.n_tokens + kScatterChunk - 1) / kScatterChunk : 1;
    return launch_pdl(route_kernel, dim3(grid), dim3(256), 0, st, a);
}

}  // namespace prism
