// tc_ffn.cu - tcgen05 row-tile GEMM chain for sm_100a.
//
// One persistent CTA per SM walks 128-row tiles.  Per tile:
//   GEMM1  acc1[128 x HID] = A[128 x KIN] . W1^T         (TMEM, fp32)
//   epi1   h = act(fp16(acc1 + b1))  -> fp16 tile H in shared memory (K-major SW128)
//   GEMM2  acc2[128 x NOUT] = H . W2^T                     (TMEM, fp32)   [two-GEMM modes]
//   epi2   the chunked dense rule (fp16 sum of chunk outputs, residual add)
// The rounding points are those of the reference shaders: every coopVecMatMulAddNV
// result is rounded to fp16 once (acc + bias), GELU is evaluated in fp32 on that
// fp16 value and rounded again, the residual add is an fp16 add.
//
// Modes: the 128<->256 adapters (one GEMM) and the dense FFN of a dense block (two GEMMs,
// NCH chunks); the grouped expert FFN has its own kernel (expert_tc.cu).
//
// Warp roles (576 threads):
//   warp 0     producer: A tile by TMA (contiguous rows) and the W1/W2 K-chunks (TMA,
//              128B swizzle) through a STAGES-deep ring
//   warp 1     TMEM allocation + single-thread tcgen05.mma issue
//   warps 2-17 epilogue (four per SM sub-partition, to hide the latency of the per-element
//              chains): warp w reads TMEM lanes 32*(w%4).. (its rows) and one quarter
//              of the columns
#include "common.cuh"
#include "tc_ffn.cuh"

namespace prism {

namespace {

constexpr int kEpiWarps = 16;                 // epilogue: 4 per SM sub-partition
constexpr int kParts = kEpiWarps / 4;          // column parts: warp 2 + 4p + q owns rows 32q.., part p
constexpr int kThreads = 32 * (2 + kEpiWarps);

template <int MODE, int KIN, int HID, int NOUT>
struct FfnCfg {
    static_assert(MODE != FFN_EXPERT, "the expert FFN is expert_tc.cu");
    static constexpr bool kTwoGemm = (MODE == FFN_DENSE || MODE == FFN_DENSE_UNSPLIT);
    static constexpr bool kUnsplit = (MODE == FFN_DENSE_UNSPLIT);  // acc2 accumulates over chunks
    static constexpr int kA = KIN * 128 * 2;                    // A tile bytes
    static constexpr int kH = kTwoGemm ? HID * 128 * 2 : 0;     // H tile bytes
    static constexpr int kWRows = HID > NOUT ? HID : NOUT;      // rows of one W K-chunk
    static constexpr int kStage = kWRows * 128;                 // bytes of one ring stage
    static constexpr int kStages = kTwoGemm ? 3 : 4;
    static constexpr int kTmemCols = kTwoGemm ? 512 : 256;
    static constexpr int kAcc2 = 256;                           // TMEM column of acc2
    static constexpr int kBarBytes = 256;
    static constexpr int kSmem = kA + kH + kStages * kStage + kBarBytes + 1024;  // + alignment slack
};

// The epilogue writes the H tile by column parts (kParts of them, each in column
// order), so K-blocks become ready part by part, interleaved; in the
// order 0, n/2, 1, n/2+1, ...; GEMM2 consumes them (and the producer loads W2) in it.
template <int HID>
__host__ __device__ constexpr int h_block_order(int i) {
    constexpr int bpp = HID / kParts / 64 > 0 ? HID / kParts / 64 : 1;  // K-blocks per column part
    return (i % kParts) * bpp + i / kParts;
}
// Warps that write one 64-column K-block of H (4 row quads x the parts it spans).
template <int HID>
__host__ __device__ constexpr int h_block_writers() {
    return HID / kParts >= 64 ? 4 : 4 * (64 / (HID / kParts));
}

struct Bars {
    uint64_t full[4], empty[4];
    uint64_t a_full, a_empty, acc1_full, acc1_empty, h_full[4], acc2_full, acc2_empty, drain;
    uint32_t tmem_base;
    int abort;
};

template <int MODE, int KIN, int HID, int NOUT>
__global__ void __launch_bounds__(kThreads, 1)
    ffn_tc_kernel(const FfnArgs a, const __grid_constant__ CUtensorMap tm_x,
                  const __grid_constant__ CUtensorMap tm_w1, const __grid_constant__ CUtensorMap tm_w2,
                  int n_chunks) {
    using Cfg = FfnCfg<MODE, KIN, HID, NOUT>;
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte alignment for the swizzled operand tiles
    unsigned char* smem = smem_align1k(smem_raw);
    unsigned char* sA = smem;
    unsigned char* sH = sA + Cfg::kA;
    unsigned char* sW = sH + Cfg::kH;
    Bars* bars = reinterpret_cast<Bars*>(sW + Cfg::kStages * Cfg::kStage);
    volatile int* abort = &bars->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles = (a.n_rows + 127) / 128;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        mbar_init(&bars->a_full, 1);
        mbar_init(&bars->a_empty, 1);  // the MMA warp's commit after the last GEMM1 reading A
        mbar_init(&bars->acc1_full, 1);
        mbar_init(&bars->acc1_empty, kEpiWarps);
        for (int kb = 0; kb < 4; ++kb) mbar_init(&bars->h_full[kb], h_block_writers<HID>());
        mbar_init(&bars->acc2_full, 1);
        mbar_init(&bars->acc2_empty, kEpiWarps);
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_barrier_init();
        fence_async_shared();
    }
    if (warp == 1) tmem_alloc(&bars->tmem_base, Cfg::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    grid_dep_wait();  // the input rows come from the previous kernel

    if (warp == 0) {
        // ===================== producer =====================
        if (lane == 0) {
            prefetch_tmap(&tm_w1);
            if (Cfg::kTwoGemm) prefetch_tmap(&tm_w2);
            prefetch_tmap(&tm_x);
        }
        int stage = 0;
        uint32_t phase = 0;
        uint32_t it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++it) {
            const int start = tile * 128;
            // --- A rows by TMA
            if (!mbar_wait(&bars->a_empty, (it & 1) ^ 1, abort)) { ok = false; break; }
            if (lane == 0) {
                mbar_expect_tx(&bars->a_full, Cfg::kA);
#pragma unroll
                for (int kb = 0; kb < KIN / 64; ++kb)
                    tma_load_2d(smem_u32(sA + kb * 16384), &tm_x, &bars->a_full, kb * 64, start);
            }
            // --- weight K-chunks, in the order the MMA warp consumes them
            for (int c = 0; c < n_chunks && ok; ++c) {
                for (int kc = 0; kc < KIN / 64; ++kc) {  // GEMM1: W1 rows of this chunk
                    if (!mbar_wait(&bars->empty[stage], phase ^ 1, abort)) { ok = false; break; }
                    if (lane == 0) {
                        mbar_expect_tx(&bars->full[stage], HID * 128);
                        tma_load_2d(smem_u32(sW + stage * Cfg::kStage), &tm_w1, &bars->full[stage], kc * 64, c * HID);
                    }
                    if (++stage == Cfg::kStages) { stage = 0; phase ^= 1; }
                }
                if (!Cfg::kTwoGemm) continue;
                for (int i = 0; i < HID / 64 && ok; ++i) {  // GEMM2: W2 columns, in H hand-off order
                    const int kc = h_block_order<HID>(i);
                    if (!mbar_wait(&bars->empty[stage], phase ^ 1, abort)) { ok = false; break; }
                    if (lane == 0) {
                        mbar_expect_tx(&bars->full[stage], NOUT * 128);
                        tma_load_2d(smem_u32(sW + stage * Cfg::kStage), &tm_w2, &bars->full[stage], c * HID + kc * 64, 0);
                    }
                    if (++stage == Cfg::kStages) { stage = 0; phase ^= 1; }
                }
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ===================== MMA issuer =====================
        // the whole warp runs this role converged; one elected lane issues
        constexpr uint32_t idesc1 = idesc_f16(128, HID);
        constexpr uint32_t idesc2 = idesc_f16(128, NOUT);
        int stage = 0;
        uint32_t phase = 0;
        uint32_t it = 0;
        uint32_t chunk_it = 0;  // counts (tile, chunk) pairs for the acc barriers
        bool ok = true;
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++it) {
            if (!mbar_wait_w(&bars->a_full, it & 1, abort)) { ok = false; break; }
            fence_async_shared();
            tc_fence_after();
            for (int c = 0; c < n_chunks && ok; ++c, ++chunk_it) {
                // GEMM1 -> acc1 (columns [0, HID))
                if (!mbar_wait_w(&bars->acc1_empty, (chunk_it & 1) ^ 1, abort)) { ok = false; break; }
                tc_fence_after();
                for (int kc = 0; kc < KIN / 64; ++kc) {
                    if (!mbar_wait_w(&bars->full[stage], phase, abort)) { ok = false; break; }
                    tc_fence_after();
                    {
                        const uint32_t a0 = smem_u32(sA + kc * 16384);
                        const uint32_t b0 = smem_u32(sW + stage * Cfg::kStage);
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            mma_f16_ss_w(tmem, sdesc(a0 + k * 32, SW128), sdesc(b0 + k * 32, SW128), idesc1,
                                         (kc | k) != 0);
                        mma_commit_w(&bars->empty[stage]);
                    }
                    if (++stage == Cfg::kStages) { stage = 0; phase ^= 1; }
                }
                if (!ok) break;
                mma_commit_w(&bars->acc1_full);
                if (c == n_chunks - 1) mma_commit_w(&bars->a_empty);  // A tile no longer needed
                if (!Cfg::kTwoGemm) continue;
                // GEMM2 -> acc2 (columns [256, 256 + NOUT)), A = H from the epilogue,
                // one K-block at a time as the epilogue hands them over
                // acc2 is handed over once per chunk, or once per tile when it accumulates over chunks
                const uint32_t acc2_it = Cfg::kUnsplit ? it : chunk_it;
                for (int i = 0; i < HID / 64; ++i) {
                    const int kc = h_block_order<HID>(i);
                    if (!mbar_wait_w(&bars->h_full[kc], chunk_it & 1, abort)) { ok = false; break; }
                    if (i == 0 && (!Cfg::kUnsplit || c == 0) &&
                        !mbar_wait_w(&bars->acc2_empty, (acc2_it & 1) ^ 1, abort)) { ok = false; break; }
                    fence_async_shared();
                    tc_fence_after();
                    if (!mbar_wait_w(&bars->full[stage], phase, abort)) { ok = false; break; }
                    tc_fence_after();
                    {
                        const uint32_t a0 = smem_u32(sH + kc * 16384);
                        const uint32_t b0 = smem_u32(sW + stage * Cfg::kStage);
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            mma_f16_ss_w(tmem + Cfg::kAcc2, sdesc(a0 + k * 32, SW128), sdesc(b0 + k * 32, SW128),
                                         idesc2, (Cfg::kUnsplit && c > 0) || (i | k) != 0);
                        mma_commit_w(&bars->empty[stage]);
                    }
                    if (++stage == Cfg::kStages) { stage = 0; phase ^= 1; }
                }
                if (!ok) break;
                if (!Cfg::kUnsplit || c == n_chunks - 1) mma_commit_w(&bars->acc2_full);
            }
        }
        // every issued MMA has completed before TMEM is released
        grid_dep_launch();  // every MMA of this CTA is issued
        mma_commit_w(&bars->drain);
        mbar_wait_w(&bars->drain, 0, abort);
    } else if (warp >= 2 && warp < 2 + kEpiWarps) {
        // ===================== epilogue =====================
        const int quad = warp & 3;               // TMEM lanes 32*quad .. +31
        const int half = (warp - 2) >> 2;        // column part (0 .. kParts-1)
        const int row = quad * 32 + lane;        // tile row of this thread
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        uint32_t it = 0, chunk_it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++it) {
            const int e = 0;
            const int start = tile * 128;
            const int rows = min(128, a.n_rows - start);
            const bool row_valid = row < rows;
            const int out_row = start + row;
            // This warp's bias columns, lane l holding columns 4l .. 4l+3 of its part (HID / kParts and
            // NOUT / 2 are 128 here); loaded as the tile starts so the L2 latency hides behind the
            // GEMM, and handed to the column groups by shuffles.
            static_assert(HID / 2 <= 128 && NOUT / 2 <= 128, "one float4 of bias per lane");
            // fp16 running sum of the dense FFN chunk outputs (attention_windowed_d256.comp.glsl:167-168)
            uint32_t accum[MODE == FFN_DENSE ? NOUT / kParts / 2 : 1];
            if (MODE == FFN_DENSE) {
#pragma unroll
                for (int i = 0; i < NOUT / kParts / 2; ++i) accum[i] = 0u;
            }
            for (int c = 0; c < n_chunks && ok; ++c, ++chunk_it) {
                // ---- epi1: acc1 -> bias -> fp16 -> activation -> fp16
                const float* b1 = a.b1 + (size_t)e * HID * n_chunks + c * HID;
                constexpr int kCols1 = HID / kParts;
                const float4 bias1 = 4 * lane < kCols1 ? ldg_f4(b1 + half * kCols1 + 4 * lane) : make_float4(0, 0, 0, 0);
                if (!mbar_wait(&bars->acc1_full, chunk_it & 1, abort)) { ok = false; break; }
                tc_fence_after();
#pragma unroll 1
                for (int g = 0; g < kCols1 / 32; ++g) {
                    const int col0 = half * kCols1 + g * 32;
                    uint32_t r[32];
                    tmem_ld32(tmem + lane_addr + col0, r);
                    tmem_ld_wait();
                    uint32_t packed[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        // columns col0 + 2j, +1 live in lane g * 8 + j / 2
                        const float bx = __shfl_sync(0xffffffffu, (j & 1) ? bias1.z : bias1.x, g * 8 + (j >> 1));
                        const float by = __shfl_sync(0xffffffffu, (j & 1) ? bias1.w : bias1.y, g * 8 + (j >> 1));
                        // t = h(acc + b1): one rounding per coopVecMatMulAddNV result
                        const uint32_t t = pack_h2(__fadd_rn(__uint_as_float(r[2 * j]), bx),
                                                   __fadd_rn(__uint_as_float(r[2 * j + 1]), by));
                        if (Cfg::kTwoGemm) {
                            packed[j] = pack_h2(gelu_f32(lo_h2f(t)), gelu_f32(hi_h2f(t)));
                        } else if (MODE == FFN_PROJ_UP) {
                            const float v0 = lo_h2f(t), v1 = hi_h2f(t);
                            packed[j] = pack_h2(v0 < 0.0f ? 0.0f : v0, v1 < 0.0f ? 0.0f : v1);
                        } else {
                            packed[j] = t;
                        }
                    }
                    if (Cfg::kTwoGemm) {
                        // H tile, K-major SW128: column col0 -> K-block col0/64, chunks (col0%64)/8 ..
                        unsigned char* blk = sH + (col0 >> 6) * 16384;
                        const int ch = (col0 & 63) >> 3;
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            *reinterpret_cast<uint4*>(blk + sw128_off(row, ch + q)) =
                                make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
                        // K-block col0/64 complete for this warp's rows (its part covers 64 columns
                        // of it, or all 32 of a 32-column part): hand it to GEMM2
                        if ((g & 1) || kCols1 == 32) {
                            fence_async_shared();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&bars->h_full[col0 >> 6]);
                        }
                    } else if (row_valid) {
                        uint4* dst = reinterpret_cast<uint4*>(a.y + (size_t)out_row * NOUT + col0);
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            dst[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->acc1_empty);
                if (!Cfg::kTwoGemm) continue;

                // ---- epi2: acc2 -> bias -> fp16 -> (+ residual) -> store.
                // The residual rows (the A tile, already released to the next gather) are
                // re-read from global memory (L2) while GEMM2 runs, and the output goes
                // out through this warp's own slice of the H tile (free once GEMM2 is
                // done): both global transfers are row-contiguous, 16 lanes per 256 B.
                const bool last = (c == n_chunks - 1);
                if (Cfg::kUnsplit && !last) continue;  // acc2 keeps accumulating over the chunks
                constexpr int kCols2 = NOUT / kParts;      // this warp's column part
                constexpr int kRowsPerLd = 512 / (kCols2 * 2);  // rows per 512-B warp access
                constexpr int kLanesPerRow = 32 / kRowsPerLd;
                constexpr int kIters = 32 / kRowsPerLd;
                const int sub_row = lane / kLanesPerRow, sub_col = (lane % kLanesPerRow) * 8;  // 8 halves / lane
                uint4 xres[Cfg::kTwoGemm ? kIters : 1];
                if (last) {
#pragma unroll
                    for (int i = 0; i < kIters; ++i) {
                        const int lr = i * kRowsPerLd + sub_row;
                        const int tk = __shfl_sync(0xffffffffu, out_row, lr);
                        const int vld = __shfl_sync(0xffffffffu, (int)row_valid, lr);
                        xres[i] = vld ? __ldg(reinterpret_cast<const uint4*>(a.x + (size_t)tk * KIN + half * kCols2 + sub_col))
                                      : make_uint4(0, 0, 0, 0);
                    }
                }
                const float* b2 = a.b2 + (size_t)e * NOUT;
                const float4 bias2 = 4 * lane < kCols2 ? ldg_f4(b2 + half * kCols2 + 4 * lane) : make_float4(0, 0, 0, 0);
                if (!mbar_wait(&bars->acc2_full, (Cfg::kUnsplit ? it : chunk_it) & 1, abort)) { ok = false; break; }
                tc_fence_after();
                // H-tile address of (tile row R, column col) in the K-major SW128 layout
                auto hslot = [&](int R, int col) -> unsigned char* {
                    return sH + (col >> 6) * 16384 + sw128_off(R, (col & 63) >> 3);
                };
                if (last) {
#pragma unroll
                    for (int i = 0; i < kIters; ++i)
                        *reinterpret_cast<uint4*>(hslot(quad * 32 + i * kRowsPerLd + sub_row, half * kCols2 + sub_col)) = xres[i];
                    __syncwarp();
                }
#pragma unroll
                for (int g = 0; g < kCols2 / 32; ++g) {
                    const int col0 = half * kCols2 + g * 32;
                    uint32_t r[32];
                    tmem_ld32(tmem + Cfg::kAcc2 + lane_addr + col0, r);
                    tmem_ld_wait();
                    uint32_t part[16];  // h(acc + b2)
                    float bxs[MODE == FFN_DENSE ? 16 : 1], bys[MODE == FFN_DENSE ? 16 : 1];  // for the dense rule
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float bx = __shfl_sync(0xffffffffu, (j & 1) ? bias2.z : bias2.x, g * 8 + (j >> 1));
                        const float by = __shfl_sync(0xffffffffu, (j & 1) ? bias2.w : bias2.y, g * 8 + (j >> 1));
                        if constexpr (MODE == FFN_DENSE) {
                            bxs[j] = bx;
                            bys[j] = by;
                        }
                        part[j] = pack_h2(__fadd_rn(__uint_as_float(r[2 * j]), bx),
                                          __fadd_rn(__uint_as_float(r[2 * j + 1]), by));
                    }
                    if (MODE == FFN_DENSE) {
                        // fp16 running sum of the chunk outputs (attention_windowed_d256.comp.glsl:167-168)
#pragma unroll
                        for (int j = 0; j < 16; ++j) accum[g * 16 + j] = hadd2_u32(accum[g * 16 + j], part[j]);
                    }
                    if (!last) continue;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        uint4* slot = reinterpret_cast<uint4*>(hslot(row, col0 + 8 * q));
                        const uint4 x = *slot;
                        const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
                        uint32_t z[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int k = 4 * q + j;
                            if (MODE == FFN_DENSE && n_chunks > 1) {
                                // out = h(acc - (n_chunks-1)*b2 + y)   (attention_windowed_d256.comp.glsl:171-177)
                                const float corr = (float)(n_chunks - 1);
                                const float bx = bxs[MODE == FFN_DENSE ? k : 0], by = bys[MODE == FFN_DENSE ? k : 0];
                                const uint32_t acc = accum[g * 16 + k];
                                z[j] = pack_h2(__fadd_rn(__fsub_rn(lo_h2f(acc), __fmul_rn(corr, bx)), lo_h2f(xs[j])),
                                               __fadd_rn(__fsub_rn(hi_h2f(acc), __fmul_rn(corr, by)), hi_h2f(xs[j])));
                            } else {
                                // one chunk: z = h(r + y), an fp16 residual add
                                z[j] = hadd2_u32(part[k], xs[j]);
                            }
                        }
                        *slot = make_uint4(z[0], z[1], z[2], z[3]);
                    }
                }
                if (last) {
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < kIters; ++i) {
                        const int lr = i * kRowsPerLd + sub_row;
                        const int tk = __shfl_sync(0xffffffffu, out_row, lr);
                        const int vld = __shfl_sync(0xffffffffu, (int)row_valid, lr);
                        const uint4 v = *reinterpret_cast<const uint4*>(hslot(quad * 32 + lr, half * kCols2 + sub_col));
                        if (vld) *reinterpret_cast<uint4*>(a.y + (size_t)tk * NOUT + half * kCols2 + sub_col) = v;
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->acc2_empty);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (bars->abort) {
        if (threadIdx.x == 0) atomicOr(a.err, ERR_TIMEOUT);
        // let any bulk copy still in flight land before the CTA exits
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 1000000ull) {
        }
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}

template <int MODE, int KIN, int HID, int NOUT>
cudaError_t launch_ffn(const FfnArgs& a, const CUtensorMap& tx, const CUtensorMap& t1, const CUtensorMap& t2,
                       int n_chunks, int grid, cudaStream_t s) {
    using Cfg = FfnCfg<MODE, KIN, HID, NOUT>;
    auto k = ffn_tc_kernel<MODE, KIN, HID, NOUT>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
    if (e != cudaSuccess) return e;
    if (grid <= 0) return cudaSuccess;
    return launch_pdl(k, dim3(grid), dim3(kThreads), Cfg::kSmem, s, a, tx, t1, t2, n_chunks);
}

}  // namespace

cudaError_t launch_ffn_dense256(const FfnArgs& a, const CUtensorMap& x, const CUtensorMap& w1, const CUtensorMap& w2,
                                int n_chunks, int grid, cudaStream_t s) {
    return launch_ffn<FFN_DENSE, 256, 256, 256>(a, x, w1, w2, n_chunks, grid, s);
}
int ffn_dense128_w1_box(int hidden, int chunk) {
    if (hidden <= 0 || chunk <= 0 || hidden % chunk) return 0;
    if (chunk == hidden) return hidden == 128 ? 128 : hidden % 256 == 0 ? 256 : 0;
    return chunk == 128 || chunk == 256 ? chunk : 0;
}

cudaError_t launch_ffn_dense128(const FfnArgs& a, const CUtensorMap& x, const CUtensorMap& w1, const CUtensorMap& w2,
                                int hidden, int chunk, int grid, cudaStream_t s) {
    const int box = ffn_dense128_w1_box(hidden, chunk);
    if (box == 0) return cudaErrorInvalidValue;
    if (chunk == hidden && hidden > 128)  // one product, hidden in 256-wide GEMM1 pieces
        return launch_ffn<FFN_DENSE_UNSPLIT, 128, 256, 128>(a, x, w1, w2, hidden / 256, grid, s);
    if (box == 128) return launch_ffn<FFN_DENSE, 128, 128, 128>(a, x, w1, w2, hidden / 128, grid, s);
    return launch_ffn<FFN_DENSE, 128, 256, 128>(a, x, w1, w2, hidden / 256, grid, s);
}
cudaError_t launch_ffn_proj_up(const FfnArgs& a, const CUtensorMap& x, const CUtensorMap& w, int grid,
                               cudaStream_t s) {
    return launch_ffn<FFN_PROJ_UP, 128, 256, 256>(a, x, w, w, 1, grid, s);
}
cudaError_t launch_ffn_proj_down(const FfnArgs& a, const CUtensorMap& x, const CUtensorMap& w, int grid,
                                 cudaStream_t s) {
    return launch_ffn<FFN_PROJ_DOWN, 256, 128, 128>(a, x, w, w, 1, grid, s);
}

}  // namespace prism
