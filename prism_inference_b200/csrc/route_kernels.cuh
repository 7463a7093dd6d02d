// route_kernels.cuh - counts -> segment offsets, tile list, token permutation.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace prism {

struct ExpertTile;

struct RouteArgs {
    const int32_t* counts;  // [n_experts] tokens per expert (the router's histogram)
    int32_t* counts_out;    // optional copy of the counts (nullable)
    int32_t* cursor;        // [n_experts] scatter cursors, zero on entry
    const int32_t* assign;  // [n_tokens] expert of each token
    int32_t* perm;          // [n_tokens] sorted row -> token
    ExpertTile* tiles;      // [max_tiles]
    int32_t* n_tiles;       // device tile count
    int n_experts, n_tokens;
    uint32_t* err;
};

// One launch: offsets, tile list and permutation.  The caller clears counts and cursor
// before the next router runs (the grouped expert kernel does it).
cudaError_t launch_route(const RouteArgs& a, cudaStream_t st);

}  // namespace prism
