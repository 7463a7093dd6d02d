// expert_tc.cu - grouped expert FFN of a Prism MoE block on the sm_100a tensor cores.
//
// For every row (token) routed to expert e (moe_expert_skip.comp.glsl:25-54):
//     h   = fp16(gelu(fp16(W1_e x + b1_e)))        (GELU in fp32 on the fp16 value)
//     out = fp16(fp16(W2_e h + b2_e) + x)          (the residual add is an fp16 add, :52)
// The reference dispatches the expert shader once per expert with an early return for
// tokens of other experts (prism_moe_bench.cpp:428-436); here the tiles of all experts run
// in one launch: a tile holds up to 128 rows of one expert (the permutation and tile list
// of route_kernels.cu), gathered from the token rows and scattered back.
//
// One persistent CTA per SM walks the tiles.  Per tile:
//   GEMM1  acc1[128 x 256] = A . W1_e^T            A = gathered rows in smem, tcgen05 SS
//   E1     h = gelu(...) packed as fp16 pairs over acc1 itself (TMEM): column part p
//          (128 columns) keeps its H K-blocks in [128p, 128p + 64), each written over
//          columns the same thread has already read
//   GEMM2  acc2[128 x 256] = H . W2_e^T            A = H from TMEM (tcgen05 TS form)
//   E2     out = fp16(fp16(acc2 + b2) + x), x (the same token rows) brought into a smem
//          staging tile by cp.async while GEMM2 runs, stored row-contiguously
// E1 and E2 are separate warp groups, so E2 of tile i runs while E1 works on tile i+1 (and
// GEMM1 of tile i+1 runs while E2 of tile i finishes): acc1 and acc2 are each single
// buffers and every hand-off is an mbarrier.  The MMA warp issues GEMM2(i) before
// GEMM1(i+1), so GEMM2 has read H (in acc1) before GEMM1(i+1) overwrites it.
//
// Warp roles (640 threads):
//   warp 0      producer: W1_e / W2_e K-chunks (TMA, 128B swizzle) through a 3-stage ring
//   warp 1      TMEM owner + tcgen05.mma issuer (converged warp, elected lane)
//   warps 2, 19 row gather: cp.async, one 512-byte token row per warp instruction, 64 rows
//               each (two warps keep twice the row loads in flight; the TMA engine is left
//               to the weight ring)
//   warps 3-10  E1: warp w reads TMEM lanes 32*(w%4).. and column part (w-3)/4
//   warps 11-18 E2: likewise with part (w-11)/4
// Every wait is bounded (common.cuh); on timeout the CTA sets the error word and winds
// down.  No TMA multicast.
#include "common.cuh"
#include "tc_ffn.cuh"

namespace prism {
namespace {

constexpr int kD = 256;                   // model / hidden width
constexpr int kE1Base = 3, kE2Base = 11;  // first warp of each epilogue group
constexpr int kGather2 = 19;              // the second row-gather warp
constexpr int kThreads = 32 * 20;
constexpr int kStage = 256 * 128;         // one W K-chunk: 256 rows x 64 columns fp16
constexpr int kStages = 3;
constexpr int kTile = 128 * kD * 2;       // a [128][256] fp16 tile as 4 K-major SW128 K-blocks
constexpr int kOffA = 0;                  // gathered rows (GEMM1's A)
constexpr int kOffO = kOffA + kTile;      // E2 staging: residual rows in, output rows out
constexpr int kOffW = kOffO + kTile;
constexpr int kOffBar = kOffW + kStages * kStage;
constexpr uint32_t kAcc1 = 0, kAcc2 = 256;

struct Bars {
    uint64_t full[kStages], empty[kStages];
    uint64_t a_full, a_empty, acc1_full, acc1_empty, h_full[4], acc2_full, acc2_empty, drain;
    uint32_t tmem_base;
    int abort;
    // bucket routing: inclusive prefix of the experts' tile counts, the rows of each expert's
    // last tile (1..128), the tile count and scan scratch
    int tinc[256];
    uint8_t last_rows[256];
    int n_tiles, wsum[8], wcnt[8];
};
constexpr int kSmem = kOffBar + (int)sizeof(Bars) + 1024;  // + alignment slack of the dynamic base
static_assert(kSmem <= 232448, "shared memory budget");

// GEMM2 consumes the H K-blocks in the order E1 completes them: part 0 writes K-blocks 0, 1
// and part 1 K-blocks 2, 3, both parts at once
PRISM_DEV constexpr int h_order(int i) { return (i & 1) * 2 + (i >> 1); }
// TMEM column of H K-block kb (32 columns = 64 fp16 K values)
PRISM_DEV constexpr uint32_t h_col(int kb) { return kAcc1 + 128u * (kb >> 1) + 32u * (kb & 1); }

// Tile i of the launch: from the route kernel's list, or (bucket routing) from the prefix of the
// experts' tile counts: expert e = the first whose inclusive prefix exceeds i.
PRISM_DEV ExpertTile tile_at(const FfnArgs& a, const Bars* bars, int i) {
    if (a.tiles) return a.tiles[i];
    int lo = 0, hi = a.n_route - 1;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (bars->tinc[mid] > i) hi = mid;
        else lo = mid + 1;
    }
    const int first = lo > 0 ? bars->tinc[lo - 1] : 0;  // the expert's first tile
    const int j = i - first;
    ExpertTile t;
    t.expert = lo;
    t.start = lo * a.perm_stride + j * 128;
    t.rows = j == bars->tinc[lo] - first - 1 ? (int)bars->last_rows[lo] : 128;
    t.pad = 0;
    return t;
}

// Bucket routing, by every CTA after the grid dependency wait: the counts -> the tile prefix
// (two-level shuffle scan over 256 entries, warps 0-7), the invariant sum(counts) == tokens
// (otherwise: no tiles and ERR_ROUTE) and the copy of the counts (CTA 0).  Every thread of the
// CTA calls it; release_counts() follows off the critical path.
PRISM_DEV int plan_buckets(const FfnArgs& a, Bars* bars) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int n = a.n_route;
    int c = 0;
    if (tid < 256) {
        c = tid < n ? a.route_counts[tid] : 0;
        int t = (c + 127) >> 7, sum = c;
        bars->last_rows[tid] = (uint8_t)(c - ((t > 0 ? t : 1) - 1) * 128);
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int tv = __shfl_up_sync(0xffffffffu, t, d), sv = __shfl_up_sync(0xffffffffu, sum, d);
            if (lane >= d) {
                t += tv;
                sum += sv;
            }
        }
        bars->tinc[tid] = t;
        if (lane == 31) {
            bars->wsum[w] = t;
            bars->wcnt[w] = sum;
        }
    }
    __syncthreads();
    if (tid < 256) {
        int off = 0;
        for (int v = 0; v < w; ++v) off += bars->wsum[v];
        bars->tinc[tid] += off;
    }
    if (blockIdx.x == 0 && a.counts_out && tid < n) a.counts_out[tid] = c;
    __syncthreads();
    if (tid == 0) {
        int tokens = 0;
        for (int v = 0; v < 8; ++v) tokens += bars->wcnt[v];
        const bool consistent = tokens == a.n_rows;
        if (!consistent && blockIdx.x == 0) atomicOr(a.err, ERR_ROUTE);
        bars->n_tiles = consistent ? bars->tinc[255] : 0;
    }
    __syncthreads();
    return bars->n_tiles;
}

// Bucket routing, one thread per CTA once plan_buckets() has returned (the CTA's reads of the
// counts are complete): the last CTA to arrive clears the counts for the next router.
PRISM_DEV void release_counts(const FfnArgs& a) {
    __threadfence();
    if (atomicAdd(a.route_done, 1u) == gridDim.x - 1) {
        for (int i = 0; i < a.n_route; ++i) a.route_counts[i] = 0;
        *a.route_done = 0;
    }
}

// staging-tile address of (tile row R, column col): K-major SW128 K-blocks of 64 columns
PRISM_DEV unsigned char* oslot(unsigned char* sO, int R, int col) {
    return sO + (col >> 6) * 16384 + sw128_off(R, (col & 63) >> 3);
}

PRISM_DEV void arrive_warp(uint64_t* bar, int lane) {
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
}

// TMEM column of H K-block kb when the E1 parts are W columns wide (each part writes its H over
// the fp32 columns it has already read: part p, 32-column group g -> 16 columns at W p + 16 g)
PRISM_DEV uint32_t h_col_w(int kb, bool narrow) { return narrow ? kAcc1 + 64u * kb : h_col(kb); }

// E1 of one tile for the calling warp: acc1 columns [W part, W part + W) of its 32 rows ->
// h = fp16(gelu(fp16(acc + b1))) (moe_expert_skip.comp.glsl:39-46) as fp16 pairs over the columns
// already read; each completed 64-column H K-block is announced on h_full.
template <int W>
PRISM_DEV bool e1_tile(const FfnArgs& a, Bars* bars, uint32_t tmem, uint32_t lane_addr, int e, int part, int lane,
                       uint32_t it, volatile int* abort) {
    // lane l holds bias columns 4l .. 4l+3 of the part, handed out by shuffles
    const float4 bias =
        4 * lane < W ? ldg_f4(a.b1 + (size_t)e * kD + part * W + 4 * lane) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (!mbar_wait_w(&bars->acc1_full, it & 1, abort)) return false;
    tc_fence_after();
#pragma unroll 1
    for (int g = 0; g < W / 32; ++g) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_addr + kAcc1 + part * W + g * 32, r);
        tmem_ld_wait();
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            // columns 32g + 2j, +1 of the part live in lane 8g + j/2
            const float bx = __shfl_sync(0xffffffffu, (j & 1) ? bias.z : bias.x, g * 8 + (j >> 1));
            const float by = __shfl_sync(0xffffffffu, (j & 1) ? bias.w : bias.y, g * 8 + (j >> 1));
            // t = h(acc + b1): one rounding per coopVecMatMulAddNV result; both columns of the pair
            // in one f32x2 instruction per step
            float s0, s1;
            f2_unpack(f2_add(f2_pack(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), f2_pack(bx, by)), s0,
                      s1);
            const uint32_t t = pack_h2(s0, s1);
            float g0, g1;
            f2_unpack(gelu_f32x2(f2_pack(lo_h2f(t), hi_h2f(t))), g0, g1);
            packed[j] = pack_h2(g0, g1);
        }
        tmem_st16(tmem + lane_addr + kAcc1 + part * W + g * 16, packed);
        if (g & 1) {  // an H K-block (64 hidden units) complete for this warp's rows
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->h_full[(part * W) / 64 + (g >> 1)]);
        }
    }
    tc_fence_before();
    return true;
}

// E2 of one tile for the calling warp: out = fp16(fp16(acc2 + b2) + x) (moe_expert_skip.comp.glsl:
// 48-52) for output columns [W part, W part + W) of its 32 rows; x (the tile's own input rows)
// comes into the staging tile by cp.async while GEMM2 runs; rows are written back
// row-contiguously (W/8 lanes per row).  acc2_done (nullable) is arrived on once acc2 is read.
template <int W>
PRISM_DEV bool e2_tile(const FfnArgs& a, Bars* bars, uint32_t tmem, uint32_t lane_addr, unsigned char* sO,
                       const ExpertTile& t, int quad, int part, int lane, uint32_t it, volatile int* abort,
                       uint64_t* acc2_done) {
    constexpr int kLanesPerRow = W / 8, kRowsPerInstr = 32 / kLanesPerRow;
    const int row = quad * 32 + lane;  // tile row of this thread (= TMEM lane)
    const int sub_row = lane / kLanesPerRow, sub_col = (lane % kLanesPerRow) * 8;
    const bool row_valid = row < t.rows;
    const int out_row = row_valid ? a.perm[t.start + row] : 0;
    // the residual rows (L2-resident) into this warp's slice of the staging tile; invalid rows
    // zero-filled
#pragma unroll
    for (int i = 0; i < 32 / kRowsPerInstr; ++i) {
        const int lr = kRowsPerInstr * i + sub_row;
        const int tk = __shfl_sync(0xffffffffu, out_row, lr);
        const int vld = __shfl_sync(0xffffffffu, (int)row_valid, lr);
        cp_async16(smem_u32(oslot(sO, quad * 32 + lr, part * W + sub_col)),
                   a.x + (size_t)(vld ? tk : 0) * kD + part * W + sub_col, vld ? 16u : 0u);
    }
    cp_async_commit();
    const float4 bias =
        4 * lane < W ? ldg_f4(a.b2 + (size_t)t.expert * kD + part * W + 4 * lane) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (!mbar_wait_w(&bars->acc2_full, it & 1, abort)) return false;
    tc_fence_after();
    cp_async_wait_all();
    __syncwarp();
#pragma unroll 1
    for (int g = 0; g < W / 32; ++g) {
        const int col0 = part * W + g * 32;
        uint32_t r[32];
        tmem_ld32(tmem + lane_addr + kAcc2 + col0, r);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint4* slot = reinterpret_cast<uint4*>(oslot(sO, row, col0 + 8 * q));
            const uint4 x = *slot;
            const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
            uint32_t z[4];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int j = 4 * q + jj;
                const float bx = __shfl_sync(0xffffffffu, (j & 1) ? bias.z : bias.x, g * 8 + (j >> 1));
                const float by = __shfl_sync(0xffffffffu, (j & 1) ? bias.w : bias.y, g * 8 + (j >> 1));
                // z = h(h(acc + b2) + x): the fp16 residual add of moe_expert_skip.comp.glsl:52
                z[jj] = hadd2_u32(pack_h2(__fadd_rn(__uint_as_float(r[2 * j]), bx), __fadd_rn(__uint_as_float(r[2 * j + 1]), by)),
                                  xs[jj]);
            }
            *slot = make_uint4(z[0], z[1], z[2], z[3]);
        }
    }
    tc_fence_before();
    if (acc2_done) arrive_warp(acc2_done, lane);  // acc2 read: GEMM2 of the next tile may go
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 32 / kRowsPerInstr; ++i) {
        const int lr = kRowsPerInstr * i + sub_row;
        const int tk = __shfl_sync(0xffffffffu, out_row, lr);
        const int vld = __shfl_sync(0xffffffffu, (int)row_valid, lr);
        const uint4 v = *reinterpret_cast<const uint4*>(oslot(sO, quad * 32 + lr, part * W + sub_col));
        if (vld) *reinterpret_cast<uint4*>(a.y + (size_t)tk * kD + part * W + sub_col) = v;
    }
    __syncwarp();  // the slice is free for the next tile's residual rows
    return true;
}

__global__ void __launch_bounds__(kThreads, 1)
    expert_tc_kernel(const FfnArgs a, const __grid_constant__ CUtensorMap tm_w1,
                     const __grid_constant__ CUtensorMap tm_w2) {
    extern __shared__ unsigned char smem_raw[];
    // (a generic base, rebuilt from an integer: measured 5 % faster for this kernel than the
    // shared-window base of smem_align1k, 0.171 against 0.180 ms per 64-frame launch, while the
    // attention and codec kernels gain from the shared window)
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    unsigned char* sA = smem + kOffA;
    unsigned char* sO = smem + kOffO;
    unsigned char* sW = smem + kOffW;
    Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
    volatile int* abort = &bars->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        mbar_init(&bars->a_full, 64);     // the gather warps' lanes, once their cp.async landed
        mbar_init(&bars->a_empty, 1);     // GEMM1 has read A (commit)
        mbar_init(&bars->acc1_full, 1);
        mbar_init(&bars->acc1_empty, 8);  // E1 has read acc1 (its H stays for GEMM2, issued first)
        for (int kb = 0; kb < 4; ++kb) mbar_init(&bars->h_full[kb], 4);  // the 4 row quads of a part
        mbar_init(&bars->acc2_full, 1);
        mbar_init(&bars->acc2_empty, 8);  // E2 has read acc2
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_barrier_init();
        fence_async_shared();
    }
    if (warp == 1) tmem_alloc(&bars->tmem_base, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    grid_dep_launch();  // the next kernel may place its CTAs (it waits for this grid to complete)
    grid_dep_wait();    // tile list, permutation and rows come from the previous kernels
    int n_tiles;
    if (a.tiles) {
        n_tiles = *a.n_tiles;
        // the routing kernel is done with the counts and cursors: clear them for the next
        // block's router (which starts only after this kernel completes)
        if (blockIdx.x == 0 && a.route_counts)
            for (int i = threadIdx.x; i < a.n_route; i += blockDim.x) {
                a.route_counts[i] = 0;
                a.route_cursor[i] = 0;
            }
    } else {
        n_tiles = plan_buckets(a, bars);
    }
    // no CTA has a second tile: the epilogues split each one over all 16 epilogue warps
    const bool single = n_tiles <= (int)gridDim.x;

    if (warp == 0) {
        // ============================ producer ============================
        if (lane == 0) {
            prefetch_tmap(&tm_w1);
            prefetch_tmap(&tm_w2);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            auto load = [&](const CUtensorMap* map, int col, int row) {
                if (!mbar_wait(&bars->empty[stage], phase ^ 1, abort)) return false;
                mbar_expect_tx(&bars->full[stage], kStage);
                tma_load_2d(smem_u32(sW + stage * kStage), map, &bars->full[stage], col, row);
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1;
                }
                return true;
            };
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                const int e = tile_at(a, bars, tile).expert;
                for (int kc = 0; kc < 4 && ok; ++kc) ok = load(&tm_w1, kc * 64, e * kD);      // W1_e
                for (int i = 0; i < 4 && ok; ++i) ok = load(&tm_w2, h_order(i) * 64, e * kD);  // W2_e
            }
        } else if (lane == 1 && !a.tiles) {
            release_counts(a);
        }
    } else if (warp == 2 || warp == kGather2) {
        // ============================ row gather ============================
        // warp 2 takes tile rows 0-63, the second warp rows 64-127; lane l copies 16-byte
        // chunk l of each row into its swizzled slot, rows past the tile are zero-filled.
        // Each lane arrives on a_full once its copies have landed.
        uint32_t it = 0;
        const uint32_t a_base = smem_u32(sA);
        const uint32_t dst_lane = a_base + (lane >> 3) * 16384;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
            const ExpertTile t = tile_at(a, bars, tile);
            const int j0 = warp == 2 ? 0 : 2;  // this warp's row blocks: j0, j0 + 1 (32 rows each)
            int tok[4];                        // token of row 32j + lane (own blocks only)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = 32 * j + lane;
                tok[j] = (j >> 1) == (j0 >> 1) && r < t.rows ? a.perm[t.start + r] : -1;
            }
            if (!mbar_wait_w(&bars->a_empty, (it & 1) ^ 1, abort)) break;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if ((j >> 1) != (j0 >> 1)) continue;
#pragma unroll 8
                for (int i = 0; i < 32; ++i) {
                    const int tk = __shfl_sync(0xffffffffu, tok[j], i);
                    const int r = 32 * j + i;
                    cp_async16(dst_lane + sw128_off(r, lane & 7), a.x + (size_t)(tk < 0 ? 0 : tk) * kD + lane * 8,
                               tk < 0 ? 0u : 16u);
                }
            }
            cp_async_mbar_arrive(&bars->a_full);
        }
    } else if (warp == 1) {
        // ============================ MMA issuer ============================
        constexpr uint32_t idesc = idesc_f16(128, 256);
        int stage = 0;
        uint32_t phase = 0;
        uint32_t it = 0;
        bool ok = true;
        auto wait = [&](uint64_t* bar, uint32_t par) {
            if (ok && !mbar_wait_w(bar, par, abort)) ok = false;
            tc_fence_after();
        };
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++it) {
            // ---- GEMM1: acc1 = A . W1^T (E1 done with the previous tile's acc1)
            wait(&bars->a_full, it & 1);
            fence_async_shared();  // the gathered rows (cp.async) are read by the tensor cores
            wait(&bars->acc1_empty, (it & 1) ^ 1);
            for (int kc = 0; kc < 4 && ok; ++kc) {
                wait(&bars->full[stage], phase);
                if (!ok) break;
                const uint32_t a0 = smem_u32(sA + kc * 16384), b0 = smem_u32(sW + stage * kStage);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    mma_f16_ss_w(tmem + kAcc1, sdesc(a0 + k * 32, SW128), sdesc(b0 + k * 32, SW128), idesc,
                                 (kc | k) != 0);
                mma_commit_w(&bars->empty[stage]);
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            mma_commit_w(&bars->acc1_full);
            mma_commit_w(&bars->a_empty);
            // ---- GEMM2: acc2 = H . W2^T, H K-blocks from TMEM as E1 hands them over
            // (E2 done with the previous tile's acc2)
            wait(&bars->acc2_empty, (it & 1) ^ 1);
            for (int i = 0; i < 4 && ok; ++i) {
                const int kb = h_order(i);
                wait(&bars->h_full[kb], it & 1);
                wait(&bars->full[stage], phase);
                if (!ok) break;
                const uint32_t b0 = smem_u32(sW + stage * kStage);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    mma_f16_ts_w(tmem + kAcc2, tmem + h_col_w(kb, single) + 8 * k, sdesc(b0 + k * 32, SW128), idesc,
                                 (i | k) != 0);
                mma_commit_w(&bars->empty[stage]);
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            mma_commit_w(&bars->acc2_full);
        }
        // every issued MMA has completed before TMEM is released
        mma_commit_w(&bars->drain);
        mbar_wait_w(&bars->drain, 0, abort);
    } else if (warp < kE2Base + 8) {
        // ============================ epilogues ============================
        // E1 (acc1 -> H) and E2 (acc2 -> out + residual) of a tile.  Normally warps 3-10 run E1 and
        // warps 11-18 E2, each warp on its TMEM row quad and a 128-column part, so E1 of tile i+1
        // runs beside E2 of tile i.  When no CTA has a second tile (a small forward: one frame is
        // ~100 tiles on 148 SMs) the two groups would take turns on the one tile, so all 16 warps
        // run E1 and then E2 on 64-column parts.
        const int quad = warp & 3;  // TMEM lanes 32*quad .. +31
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        if (single) {
            const int part = (warp - kE1Base) >> 2;  // columns [64 part, 64 part + 64)
            if ((int)blockIdx.x < n_tiles) {
                const ExpertTile t = tile_at(a, bars, blockIdx.x);
                if (e1_tile<64>(a, bars, tmem, lane_addr, t.expert, part, lane, 0u, abort) && warp < kE2Base)
                    arrive_warp(&bars->acc1_empty, lane);
                e2_tile<64>(a, bars, tmem, lane_addr, sO, t, quad, part, lane, 0u, abort,
                            warp >= kE2Base ? &bars->acc2_empty : nullptr);
            }
        } else if (warp < kE2Base) {
            const int part = (warp - kE1Base) >> 2;  // columns [128 part, 128 part + 128)
            uint32_t it = 0;
            for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
                if (!e1_tile<128>(a, bars, tmem, lane_addr, tile_at(a, bars, tile).expert, part, lane, it, abort)) break;
                arrive_warp(&bars->acc1_empty, lane);
            }
        } else {
            const int part = (warp - kE2Base) >> 2;
            uint32_t it = 0;
            for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
                if (!e2_tile<128>(a, bars, tmem, lane_addr, sO, tile_at(a, bars, tile), quad, part, lane, it, abort,
                                  &bars->acc2_empty))
                    break;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (bars->abort) {
        if (threadIdx.x == 0) atomicOr(a.err, ERR_TIMEOUT);
        // let any copy still in flight land before the CTA exits
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 1000000ull) {
        }
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace

cudaError_t launch_ffn_expert256(const FfnArgs& a, const CUtensorMap& w1, const CUtensorMap& w2, int grid,
                                 cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(expert_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    if (grid <= 0) return cudaSuccess;
    return launch_pdl(expert_tc_kernel, dim3(grid), dim3(kThreads), kSmem, s, a, w1, w2);
}

}  // namespace prism
