// codec_tc.cu - the encoder / decoder passes around the transformer stack, on the sm_100a
// tensor cores: the 540p -> 1080p frame path of prism_moe_bench.cpp:386-471 without the stack.
//
// Eight of the nine shaders are contractions of a per-pixel input vector with a fixed weight
// matrix, as coopVecMatMulAddNV products:
//   conv3x3_coopvec_9ch        9 -> 32, 3x3 stride 1 (K = 81), ReLU by push constant
//   strided_conv_coopvec_32ch  32 -> 64, 3x3 stride 2 (K = 288), ReLU
//   strided_conv_split_64ch    64 -> 128, stride 2, two 32-channel groups (K = 288 each): the two
//                              products, each rounded to fp16, summed in fp32 minus one bias, ReLU
//   strided_conv_split_128ch   128 -> 128, stride 2, four groups: fp16 running sum of the group
//                              products with the bias removed per group, ReLU
//   dec3 / dec2 / dec1_fused   nearest 2x upsample of the deeper map (clamped to its edge)
//                              concatenated with the skip map, pointwise product, ReLU
//   pw_conv_coopvec_32to12     32 -> 12 pointwise, ReLU by push constant
// Each runs here as an implicit GEMM: a tile is 128 output pixels (rows = MMA M), N = output
// channels, K = the shader's input vector (channel, ky, kx order; tap-major for the 3x3
// convolutions), one TMEM accumulator per channel group.  Feature maps are CHW fp16 at element
// offsets of the caller's arena.  Weight matrices of up to 64 KB are built in shared memory from
// the blob once per CTA (SW128 K-blocks); the two split convolutions' matrices are repacked by a
// small kernel into an aligned K-major copy that a ring streams by TMA.
// The ninth shader, pixelshuffle_sigmoid, is elementwise (SIMT kernel at the end of the file).
//
// Two forms of the contraction kernel:
//   plain   tiles of 128 consecutive pixels of the map; the gather warps load the patch values
//           with per-lane 16-bit loads (any alignment; zero outside the map)
//   staged  (conv3x3_9ch, dec2, dec1, pointwise, when the maps' bases and row pitches are
//           16-byte multiples) tiles of 128 pixels of one output row; the producer brings each
//           tile's input rows into shared memory by TMA (3-D boxes {x, y, channel}; the zero fill
//           outside the map is the padding), 2 to 8 tiles ahead; the gather warps build the A
//           tile from there (dec / pointwise: 64-pixel 128B-swizzled rows, transposed 8 x 8 at a
//           time by ldmatrix.trans + stmatrix); two epilogue groups take alternate tiles (one TMEM accumulator
//           buffer each) and stage their output tiles in shared memory for one TMA store each
//           (clipped at the map's edge).  The per-tile epilogue chain (TMEM load, bias, fp16,
//           ReLU, stores) is what bounds these passes; the second group and the bulk stores
//           halve its share.  dec3 (plain form) takes the two epilogue groups as well.
//
// Warp roles (448 threads; 576 with two epilogue groups):
//   warp 0      producer: staged input rows by TMA; streamed weight K-blocks {64 K, N rows}
//               (128B swizzle, no multicast)
//   warp 1      TMEM owner + tcgen05.mma issuer
//   warps 2-9   gather: warp 2 + 4h + q fills rows 32q.. with K columns [32h, 32h + 32) of every
//               K-block, 16-byte stores into the swizzled A tile
//   warps 10-13 epilogue: TMEM -> the shader's rounding / group rule -> CHW output (direct
//   (+14-17)    stores: each warp instruction writes 32 consecutive pixels of one channel)
// The A K-blocks pass through a ring of 8 stages where shared memory allows (6 for dec2 and dec3,
// beside their weights and staging tiles; 4 with streamed weights, whose B K-blocks share the
// stage).  Every wait is bounded (common.cuh); on timeout the CTA sets the context's error word and
// winds down.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "host_util.h"

namespace prism {
namespace {

// kinds in the order of prism_codec_kind (include/prism_moe.h)
enum : int { C_ENC_IC = 0, C_ENC1, C_ENC2, C_ENC3, C_DEC3, C_DEC2, C_DEC1, C_OUT12, C_PS, C_COUNT };

constexpr int kMaxStages = 8;
constexpr int kMaxStg = 8;  // staging buffers (staged form)

struct Bars {
    uint64_t a_full[kMaxStages], b_full[kMaxStages], empty[kMaxStages];
    uint64_t acc_full[2], acc_empty[2], drain, stg_full[kMaxStg], stg_empty[kMaxStg], out_full[2], out_free[2];
    uint32_t tmem_base;
    int abort;
    alignas(8) float bias[128];  // (read as float2 pairs)
};

// STG: the staged form of a pass whose input is plain row segments (conv3x3_coopvec_9ch, the
// three decoder passes, the pointwise output): tiles are 128 pixels of one output row and the
// producer brings each tile's input rows into shared memory by TMA (3-D boxes {x, y, channel} of
// the CHW maps; the zero fill outside the map is the convolution's padding), two tiles ahead of
// the gather warps, which then build the A tile from shared memory.  As many staging buffers as
// shared memory holds (up to 8) keep that many tiles' row loads in flight, which is what a pass
// of ~0.5 us tiles needs against a ~2 us load latency.
template <int KIND, bool STG = false>
struct CodecCfg {
    static constexpr int kType = KIND <= C_ENC3 ? 0 : KIND <= C_DEC1 ? 1 : 2;  // conv3x3, dec, pointwise
    static constexpr int kStride = KIND == C_ENC_IC ? 1 : 2;  // of the 3x3 convolutions
    static constexpr int kIn = KIND == C_ENC_IC ? 9 : KIND == C_ENC1 ? 32 : KIND == C_ENC2 ? 64 : KIND == C_ENC3 ? 128
                                                                                                  : 32;  // conv / pw
    static constexpr int kUp = KIND == C_DEC1 ? 64 : 128;                                          // dec: deeper map
    static constexpr int kSkip = KIND == C_DEC3 ? 128 : KIND == C_DEC2 ? 64 : 32;                   // dec: skip map
    static constexpr int kN = KIND == C_ENC_IC || KIND == C_DEC1 ? 32
                              : KIND == C_ENC1 || KIND == C_DEC2 ? 64
                              : KIND == C_OUT12                 ? 12
                                                                : 128;
    static constexpr int kNP = (kN + 15) / 16 * 16;             // MMA N (multiple of 16)
    static constexpr int kG = KIND == C_ENC2 ? 2 : KIND == C_ENC3 ? 4 : 1;  // channel groups
    static constexpr int kCg = kIn / kG;                        // conv: input channels per group
    // K of one group in the blob (the shader's order: channel, then ky, then kx)
    static constexpr int kKsrc = kType == 0 ? kCg * 9 : kType == 1 ? kUp + kSkip : kIn;
    static constexpr int kLd = kG * kKsrc;                      // row stride of the blob's matrix
    // The GEMM's K order for the 3x3 convolutions is tap-major (k = tap * kCgP + channel), so one
    // 32-value half of a K-block is one tap (or two taps of 16 channel slots when a group has 9
    // channels): the gather checks bounds once per half and steps through the channel planes.
    static constexpr int kCgP = kCg >= 32 ? 32 : 16;
    static constexpr int kKG = kType == 0 ? 9 * kCgP : kKsrc;   // GEMM K per group
    static constexpr int kKGP = (kKG + 63) / 64 * 64;           // padded to whole K-blocks
    static constexpr int kKB = kKGP / 64;
    static constexpr int kAccCols = kG * kNP;
    static constexpr int kAccBufs = kAccCols <= 256 ? 2 : 1;    // TMEM accumulator buffers
    static constexpr int kBBytes = kNP * 128;                   // one weight K-block
    static constexpr int kWBytes = kG * kKB * kBBytes;          // the whole repacked weight matrix
    // Weights of up to 64 KB stay in shared memory for the whole CTA (loaded once); larger ones
    // (the split convolutions) stream through the ring beside the A K-blocks.
    static constexpr bool kResident = kWBytes <= 65536;
    // (dec3's staging buffers would not fit beside its 64 KB of weights and output staging)
    static constexpr bool kCanStage = KIND == C_ENC_IC || KIND == C_DEC2 || KIND == C_DEC1 || KIND == C_OUT12;
    // staged input of one tile: conv3x3_9ch rows y-1..y+1 of all channels, x from x0 - 8 (the
    // TMA start is 16-byte aligned) over 144 pixels, no swizzle; dec: one row of the deeper map
    // (64 pixels from x0 / 2) and of the skip map (two 64-pixel boxes); pointwise: one row (two
    // 64-pixel boxes); the dec / pointwise boxes are 128B-swizzled [channel][64 pixels] tiles
    static constexpr int kStgUp = kType == 1 ? kUp * 64 * 2 : 0;
    static constexpr int kStgBytes = !STG ? 0 : kType == 0 ? kIn * 3 * 144 * 2 : kType == 1 ? kStgUp + kSkip * 128 * 2
                                                                                              : kIn * 128 * 2;
    static constexpr int kStgBuf = (kStgBytes + 1023) / 1024 * 1024;
    static constexpr int kWRes = kResident ? (kWBytes + 1023) / 1024 * 1024 : 0;
    // epilogue groups of four warps: two take alternate tiles (one TMEM accumulator buffer each)
    // in the staged form and for dec3 (576 threads cap a thread at 96 registers: the plain-load
    // gathers of the strided convolutions then spill and ran 20-25 % slower with two groups)
    static constexpr int kEpiGroups = kAccBufs == 2 && (STG || KIND == C_DEC3) ? 2 : 1;
    static constexpr int kThreads = 32 * (10 + 4 * kEpiGroups);
    // output staging (two epilogue groups): a tile of [kN channels][128 pixels] per group, written
    // by one TMA store.  (With one group the TMA hand-off lengthens the per-tile chain: direct
    // stores measured faster there, and the plain-load gather keeps the L1 this would take.)
    static constexpr int kOutBuf = kEpiGroups == 2 ? (kN * 256 + 1023) / 1024 * 1024 : 0;
    static constexpr int kReserve = 2 * kOutBuf + (int)sizeof(Bars) + 1024;
    // A ring: 8 stages where they fit (the per-stage round trip gather -> MMA -> release bounds a
    // shallow ring), beside at least two staging buffers in the staged form
    static constexpr int kFixed = kWRes + kReserve + (STG ? 2 * kStgBuf : 0);
    static constexpr int kStages = !kResident ? 4 : 8 * 16384 + kFixed <= 232448 ? 8 : 6 * 16384 + kFixed <= 232448 ? 6 : 4;
    static constexpr int kStageBytes = kResident ? 16384 : 32768;  // A (+ B when streamed)
    static constexpr int kWOff = kStages * kStageBytes;         // resident weights
    static constexpr int kStgOff = kWOff + kWRes;               // the input staging buffers
    static constexpr int kStgFit = !STG ? 0 : (232448 - kReserve - kStgOff) / kStgBuf;
    static constexpr int kStgN = kStgFit > kMaxStg ? kMaxStg : kStgFit;
    static constexpr int kOutOff = kStgOff + kStgN * kStgBuf;
    static constexpr int kBarOff = kOutOff + 2 * kOutBuf;
};

constexpr int kABytes = 128 * 128;  // one A K-block: 128 rows x 64 fp16, SW128

struct CodecArgs {
    const __half* in;    // conv / pw: the input map; dec: the deeper map (CHW)
    const __half* skip;  // dec: the skip map at the output resolution (CHW)
    __half* out;         // the output map (CHW)
    int in_w, in_h, out_w, out_h;
    int relu;            // conv3x3_9ch / pw: the push constant (1 = ReLU)
    const __half* blob;  // the weights arena: matrix at element wo, biases at bo (any alignment)
    int wo, bo;
    int tma_out;         // 1: output tiles staged in shared memory and written by TMA (tm_out)
    uint32_t* err;
};

template <int KIND, bool STG>
constexpr int codec_smem() {  // + alignment slack of the dynamic base
    return CodecCfg<KIND, STG>::kBarOff + (int)sizeof(Bars) + 1024;
}

PRISM_DEV uint16_t h_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }
PRISM_DEV float bits_h(uint16_t b) { return __half2float(__ushort_as_half(b)); }
// `if (v < 0) v = 0` on an fp16 value (negative zero stays, as in the shaders)
PRISM_DEV uint16_t relu_bits(uint16_t b) { return bits_h(b) < 0.0f ? (uint16_t)0 : b; }

template <int KIND, bool STG>
__global__ void __launch_bounds__(CodecCfg<KIND, STG>::kThreads, 1)
    codec_tc_kernel(const CodecArgs a, const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_in, const __grid_constant__ CUtensorMap tm_skip,
                    const __grid_constant__ CUtensorMap tm_out) {
    using C = CodecCfg<KIND, STG>;
    static_assert(!STG || (C::kCanStage && C::kResident && C::kG == 1 && C::kStgN >= 2), "staged form");
    constexpr int kStages = C::kStages, kStageBytes = C::kStageBytes;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = smem_align1k(smem_raw);
    Bars* bars = reinterpret_cast<Bars*>(smem + C::kBarOff);
    volatile int* abort = &bars->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int out_px = a.out_w * a.out_h;
    // staged: out_h rows of tpr tiles (128 pixels of one row each); else 128 consecutive pixels
    const int tpr = (a.out_w + 127) >> 7;
    const int n_tiles = STG ? a.out_h * tpr : (out_px + 127) >> 7;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars->a_full[s], 8);  // the eight gather warps
            mbar_init(&bars->b_full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->acc_full[b], 1);
            mbar_init(&bars->acc_empty[b], 4);
        }
        mbar_init(&bars->drain, 1);
        for (int b = 0; b < C::kStgN; ++b) {
            mbar_init(&bars->stg_full[b], 1);
            mbar_init(&bars->stg_empty[b], 8);  // the eight gather warps
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->out_full[b], 4);  // the four epilogue warps have written the tile
            mbar_init(&bars->out_free[b], 1);  // its previous TMA store has read the buffer
        }
        bars->abort = 0;
        fence_barrier_init();
    }
    for (int i = threadIdx.x; i < 128; i += blockDim.x) bars->bias[i] = i < C::kN ? __half2float(a.blob[a.bo + i]) : 0.0f;
    if constexpr (C::kResident) {
        // The whole weight matrix into shared memory, straight from the blob: [g][kb] K-blocks of
        // {kNP rows, 64 K values} in the MMA's SW128 layout, K in the GEMM's order (tap-major for the
        // 3x3 convolutions: k = tap * kCgP + channel), zero padding.  Every thread builds 16-byte
        // chunks; weights are never written by a pass, so this runs before the wait for the
        // previous kernel and overlaps its end.
        constexpr int kChunks = C::kG * C::kKB * C::kNP * 8;
        for (int ci = threadIdx.x; ci < kChunks; ci += blockDim.x) {
            const int chunk = ci & 7, n = (ci >> 3) % C::kNP, gk = (ci >> 3) / C::kNP;  // gk = g * kKB + kb
            const int g = gk / C::kKB, kb = gk % C::kKB;
            uint32_t w4[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint32_t pair = 0;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int k = kb * 64 + chunk * 8 + 2 * q + h;
                    int src = -1;  // element of the group's row in the blob's (channel, tap) order
                    if (C::kType == 0) {
                        const int t = k / C::kCgP, c = k % C::kCgP;
                        if (t < 9 && c < C::kCg) src = c * 9 + t;
                    } else if (k < C::kKG) {
                        src = k;
                    }
                    if (n < C::kN && src >= 0)
                        pair |= (uint32_t)__half_as_ushort(a.blob[a.wo + (size_t)n * C::kLd + g * C::kKsrc + src]) << (16 * h);
                }
                w4[q] = pair;
            }
            *reinterpret_cast<uint4*>(smem + C::kWOff + gk * C::kBBytes + sw128_off(n, chunk)) =
                make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
        fence_async_shared();  // read by the tensor cores
    }
    if (warp == 1) tmem_alloc(&bars->tmem_base, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Programmatic dependent launch: the next pass may place its CTAs now; this one waits for the
    // previous kernels (its input maps, the repacked weights of a streamed matrix, and the
    // memory its output overwrites) only here, after the prologue above.
    grid_dep_launch();
    grid_dep_wait();
    const uint32_t tmem = bars->tmem_base;
    auto stage_a = [&](int s) { return smem + s * kStageBytes; };
    // weight K-block (g, kb) of `stage`: resident copy, or the stage's B slot when streamed
    auto b_block = [&](int s, int g, int kb) {
        return C::kResident ? smem + C::kWOff + (g * C::kKB + kb) * C::kBBytes : smem + s * kStageBytes + kABytes;
    };

    if (warp == 0) {
        // ============================ producer ============================
        if (STG && lane == 0) {  // each tile's input rows, kStgN tiles ahead of the gather
            prefetch_tmap(&tm_in);
            if (C::kType == 1) prefetch_tmap(&tm_skip);
            int b = 0;
            uint32_t bph = 0;
            for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
                if (!mbar_wait(&bars->stg_empty[b], bph ^ 1, abort)) break;
                const int oy = tile / tpr, x0 = (tile - oy * tpr) * 128;
                uint64_t* bar = &bars->stg_full[b];
                const uint32_t dst = smem_u32(smem + C::kStgOff + b * C::kStgBuf);
                mbar_expect_tx(bar, C::kStgBytes);
                if (C::kType == 0) {
                    tma_load_3d(dst, &tm_in, bar, x0 - 8, oy - 1, 0);
                } else if (C::kType == 1) {  // 64-pixel SW128 boxes: the deeper row, two skip halves
                    tma_load_3d(dst, &tm_in, bar, x0 >> 1, min(oy >> 1, a.in_h - 1), 0);
                    tma_load_3d(dst + C::kStgUp, &tm_skip, bar, x0, oy, 0);
                    tma_load_3d(dst + C::kStgUp + C::kSkip * 128, &tm_skip, bar, x0 + 64, oy, 0);
                } else {
                    tma_load_3d(dst, &tm_in, bar, x0, oy, 0);
                    tma_load_3d(dst + C::kIn * 128, &tm_in, bar, x0 + 64, oy, 0);
                }
                if (++b == C::kStgN) {
                    b = 0;
                    bph ^= 1;
                }
            }
        }
        if (lane == 0 && !C::kResident) {  // the streamed weight K-blocks beside the A K-blocks
            prefetch_tmap(&tm_w);
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x)
                for (int g = 0; g < C::kG && ok; ++g)
                    for (int kb = 0; kb < C::kKB && ok; ++kb) {
                        if (!mbar_wait(&bars->empty[s], ph ^ 1, abort)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(&bars->b_full[s], C::kBBytes);
                        tma_load_2d(smem_u32(b_block(s, g, kb)), &tm_w, &bars->b_full[s], kb * 64, g * C::kNP);
                        if (++s == kStages) {
                            s = 0;
                            ph ^= 1;
                        }
                    }
        }
    } else if (warp == 1) {
        // ============================ MMA issuer ============================
        constexpr uint32_t idesc = idesc_f16(128, C::kNP);
        int s = 0;
        uint32_t ph = 0, it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++it) {
            const int buf = C::kAccBufs == 2 ? (int)(it & 1) : 0;
            const uint32_t use = C::kAccBufs == 2 ? (it >> 1) : it;  // uses of this buffer so far
            if (!mbar_wait_w(&bars->acc_empty[buf], (use & 1) ^ 1, abort)) break;
            tc_fence_after();
            for (int g = 0; g < C::kG && ok; ++g)
#pragma unroll 1
                for (int kb = 0; kb < C::kKB; ++kb) {
                    if (!mbar_wait_w(&bars->a_full[s], ph, abort) ||
                        (!C::kResident && !mbar_wait_w(&bars->b_full[s], ph, abort))) {
                        ok = false;
                        break;
                    }
                    fence_async_shared();  // the gathered rows are read by the tensor core
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(stage_a(s)), b0 = smem_u32(b_block(s, g, kb));
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        mma_f16_ss_w(tmem + buf * 256 + g * C::kNP, sdesc(a0 + k * 32, SW128), sdesc(b0 + k * 32, SW128),
                                     idesc, (kb | k) != 0);
                    mma_commit_w(&bars->empty[s]);
                    if (++s == kStages) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            mma_commit_w(&bars->acc_full[buf]);
        }
        mma_commit_w(&bars->drain);
        mbar_wait_w(&bars->drain, 0, abort);
    } else if (STG && warp < 10) {
        // ============================ gather (staged input) ============================
        // warp 2 + 4h + q fills rows 32q.. with K columns [32h, 32h + 32) of every K-block, read
        // from the tile's staging buffer (lanes = consecutive pixels: conflict-free 16-bit reads)
        const int gw = warp - 2, quad = gw & 3, half = gw >> 2;
        const int row = quad * 32 + lane;
        int s = 0, b = 0;
        uint32_t ph = 0, bph = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
            const int oy = tile / tpr, x0 = (tile - oy * tpr) * 128;
            if (!mbar_wait(&bars->stg_full[b], bph, abort)) break;
            const unsigned short* sg = reinterpret_cast<const unsigned short*>(smem + C::kStgOff + b * C::kStgBuf);
#pragma unroll 1
            for (int kb = 0; kb < C::kKB; ++kb) {
                const int k0 = kb * 64 + half * 32;
                uint32_t w[16];
                if constexpr (C::kType == 0) {
                    // taps k0 / 16 and k0 / 16 + 1 (16 channel slots each, channels 0..8 real)
#pragma unroll
                    for (int tt = 0; tt < 2; ++tt) {
                        const int t = k0 / C::kCgP + tt;
                        const int base = (t / 3) * 144 + row + t % 3 + 7;  // x - (x0 - 8) = row + dx - 1 + 8
#pragma unroll
                        for (int c = 0; c < 16; c += 2) {
                            const uint32_t v0 = t < 9 && c < C::kIn ? sg[c * 432 + base] : 0u;
                            const uint32_t v1 = t < 9 && c + 1 < C::kIn ? sg[(c + 1) * 432 + base] : 0u;
                            w[tt * 8 + c / 2] = v0 | (v1 << 16);
                        }
                    }
                } else {
                    // dec / pointwise: 8 x 8 blocks (8 pixels x 8 channels) transposed from the
                    // staged [channel][64 pixels] SW128 rows by ldmatrix.trans (lane 8i + k: row k of
                    // block i = channel c0 + 8i + k; its eight channel rows sit in eight different
                    // bank groups); they go to the A rows by stmatrix after the stage is free
                    const uint32_t sgb = smem_u32(sg);
                    const int bi = lane >> 3, bk = lane & 7;
                    if (k0 >= C::kKG) {  // K padding
#pragma unroll
                        for (int j = 0; j < 16; ++j) w[j] = 0u;
                    } else if (C::kType == 1 && k0 < C::kUp) {
                        // the deeper map, nearest: output pixel r reads up pixel r / 2 of the row
                        // (x0 is even; rows past out_w are never stored, so no clamp is needed where
                        // out_w <= 2 in_w, which the host requires of this form)
                        const int c = k0 + 8 * bi + bk;
#pragma unroll
                        for (int ub = 0; ub < 2; ++ub) {
                            const int uc = 2 * quad + ub;  // 8-pixel chunk of the deeper row
                            ldsm_x4_trans(sgb + c * 128 + ((uc ^ (c & 7)) << 4), w[4 * ub], w[4 * ub + 1],
                                          w[4 * ub + 2], w[4 * ub + 3]);
                        }
                    } else {
                        constexpr int kC = C::kType == 1 ? C::kSkip : C::kIn;
                        const int c = k0 - (C::kType == 1 ? C::kUp : 0) + 8 * bi + bk;
#pragma unroll
                        for (int pb = 0; pb < 4; ++pb) {
                            const int r0 = 32 * quad + 8 * pb, pc = (r0 & 63) >> 3;
                            ldsm_x4_trans(sgb + C::kStgUp + (r0 >> 6) * (kC * 128) + c * 128 + ((pc ^ (c & 7)) << 4),
                                          w[4 * pb], w[4 * pb + 1], w[4 * pb + 2], w[4 * pb + 3]);
                        }
                    }
                }
                if (!mbar_wait(&bars->empty[s], ph ^ 1, abort)) {
                    ok = false;
                    break;
                }
                unsigned char* dst = stage_a(s);
                if constexpr (C::kType == 0) {
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        *reinterpret_cast<uint4*>(dst + sw128_off(row, half * 4 + c)) =
                            make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
                } else {
                    // block i of each stmatrix -> A chunk 4 half + i of eight consecutive rows
                    const uint32_t ab = smem_u32(dst);
                    const int bi = lane >> 3, bk = lane & 7;
                    if (C::kType == 1 && k0 < C::kUp && k0 < C::kKG) {
#pragma unroll
                        for (int ub = 0; ub < 2; ++ub)
#pragma unroll
                            for (int odd = 0; odd < 2; ++odd) {  // each up pixel feeds two output rows
                                const int r = 32 * quad + 16 * ub + 2 * bk + odd;
                                stsm_x4(ab + sw128_off(r, 4 * half + bi), w[4 * ub], w[4 * ub + 1], w[4 * ub + 2],
                                        w[4 * ub + 3]);
                            }
                    } else {
#pragma unroll
                        for (int pb = 0; pb < 4; ++pb)
                            stsm_x4(ab + sw128_off(32 * quad + 8 * pb + bk, 4 * half + bi), w[4 * pb], w[4 * pb + 1],
                                    w[4 * pb + 2], w[4 * pb + 3]);
                    }
                }
                fence_async_shared();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->a_full[s]);
                if (++s == kStages) {
                    s = 0;
                    ph ^= 1;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->stg_empty[b]);  // this warp is done with the buffer
            if (++b == C::kStgN) {
                b = 0;
                bph ^= 1;
            }
        }
    } else if (warp < 10) {
        // ============================ gather ============================
        // The values are fp16 already and go to the A tile unchanged, so each lane issues its 32
        // raw 16-bit loads of a K-block without branches (an address outside the map or the
        // padding reads element 0 of the map and is then replaced by zero) and keeps the next
        // K-block's loads in flight while it stores the current one.
        const int gw = warp - 2, quad = gw & 3, half = gw >> 2;
        const int row = quad * 32 + lane;
        const int in_px = a.in_w * a.in_h;
        const unsigned short* in = reinterpret_cast<const unsigned short*>(a.in);
        const unsigned short* skip = reinterpret_cast<const unsigned short*>(a.skip);
        constexpr int kItems = C::kG * C::kKB;  // K-blocks per tile
        // issue the loads of the 32 values of K-block `item` of `tile` into r; bit j of the result
        // says whether value j is real (else the shader reads zero there, and nothing is loaded)
        auto issue = [&](int tile, int item, uint32_t (&r)[32]) -> uint32_t {
            const int g = item / C::kKB, kb = item % C::kKB;
            const int p = tile * 128 + row;
            if (p >= out_px) return 0u;
            const int oy = p / a.out_w, ox = p % a.out_w;
            if constexpr (C::kType == 0) {
                const unsigned short* base = in + (int64_t)g * C::kCg * in_px;
                uint32_t mask = 0;
#pragma unroll
                for (int tt = 0; tt < 32 / C::kCgP; ++tt) {  // the taps of this half
                    const int t = (kb * 64 + half * 32) / C::kCgP + tt;
                    const int y = oy * C::kStride + t / 3 - 1, x = ox * C::kStride + t % 3 - 1;
                    if (t < 9 && y >= 0 && y < a.in_h && x >= 0 && x < a.in_w) {
                        const unsigned short* q = base + (int64_t)y * a.in_w + x;
#pragma unroll
                        for (int c = 0; c < (C::kCg < C::kCgP ? C::kCg : C::kCgP); ++c)
                            r[tt * C::kCgP + c] = __ldg(q + (int64_t)c * in_px);
                        mask |= (C::kCg < C::kCgP ? (1u << C::kCg) - 1u : 0xffffffffu) << (tt * C::kCgP);
                    }
                }
                return mask;
            } else {
                const int k0 = kb * 64 + half * 32;  // one map per half: up / skip / pointwise input
                if (k0 >= C::kKG) return 0u;
                const unsigned short* q;
                int64_t plane;
                if (C::kType == 1 && k0 < C::kUp) {
                    q = in + (int64_t)k0 * in_px + min(oy >> 1, a.in_h - 1) * a.in_w + min(ox >> 1, a.in_w - 1);
                    plane = in_px;
                } else {
                    q = (C::kType == 1 ? skip + (int64_t)(k0 - C::kUp) * out_px : in + (int64_t)k0 * out_px) + p;
                    plane = out_px;
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) r[j] = __ldg(q + j * plane);
                return 0xffffffffu;
            }
        };
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        uint32_t cur[32], nxt[32], m_cur = 0, m_nxt = 0;
        int tile = blockIdx.x, item = 0;
        if (tile < n_tiles) m_cur = issue(tile, 0, cur);
        while (tile < n_tiles && ok) {
            int nt = tile, ni = item + 1;
            if (ni == kItems) {
                ni = 0;
                nt += gridDim.x;
            }
            if (nt < n_tiles) m_nxt = issue(nt, ni, nxt);
            if (!mbar_wait(&bars->empty[s], ph ^ 1, abort)) {
                ok = false;
                break;
            }
            unsigned char* dst = stage_a(s);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t w4[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int j = 8 * c + 2 * q;
                    w4[q] = ((m_cur >> j) & 1u ? cur[j] : 0u) | ((m_cur >> (j + 1)) & 1u ? cur[j + 1] << 16 : 0u);
                }
                *reinterpret_cast<uint4*>(dst + sw128_off(row, half * 4 + c)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
            fence_async_shared();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->a_full[s]);
            if (++s == kStages) {
                s = 0;
                ph ^= 1;
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) cur[j] = nxt[j];
            m_cur = m_nxt;
            tile = nt;
            item = ni;
        }
    } else {
        // ============================ epilogue ============================
        // With tma_out, each tile's output goes to a shared-memory tile [channel][128 pixels] (a
        // thread per pixel: conflict-free 16-bit stores) that one TMA store writes to the CHW map,
        // clipped at the map's edge; two such tiles alternate.  Otherwise 16-bit global stores.
        const bool tma_out = C::kOutBuf > 0 && a.tma_out;  // (staging exists only with two groups)
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const int eg = (warp - 10) >> 2;            // epilogue group: tiles it = eg, eg + kEpiGroups, ..
        const int store_warp = 10 + 4 * eg;          // its lane 0 issues the group's TMA stores
        const bool issuer = warp == store_warp && lane == 0;
        constexpr int kChunk = C::kNP >= 32 && C::kG == 1 ? 32 : 16;  // columns per TMEM load and group
        uint32_t it = eg;
        for (int tile = blockIdx.x + eg * gridDim.x; tile < n_tiles; tile += C::kEpiGroups * gridDim.x, it += C::kEpiGroups) {
            const int buf = C::kAccBufs == 2 ? (int)(it & 1) : 0;
            const uint32_t use = C::kAccBufs == 2 ? (it >> 1) : it;
            const int ob_i = it & 1;
            const uint32_t ob_use = it >> 1;
            unsigned short* ob = reinterpret_cast<unsigned short*>(smem + C::kOutOff + ob_i * C::kOutBuf);
            if (tma_out && ob_use > 0) {
                if (issuer) {  // the store of two tiles ago has read this buffer
                    if (C::kEpiGroups == 2) tma_store_wait_read<0>();  // (the group's only buffer)
                    else tma_store_wait_read<1>();
                    mbar_arrive(&bars->out_free[ob_i]);
                }
                if (!mbar_wait_w(&bars->out_free[ob_i], (ob_use - 1) & 1, abort)) break;
            }
            if (!mbar_wait_w(&bars->acc_full[buf], use & 1, abort)) break;
            tc_fence_after();
            int p, sx, sy;  // pixel index; the tile's TMA store coordinates
            bool valid;
            if constexpr (STG) {
                const int oy = tile / tpr, x0 = (tile - oy * tpr) * 128;
                p = oy * a.out_w + x0 + row;
                valid = x0 + row < a.out_w;
                sx = x0, sy = oy;
            } else {
                p = tile * 128 + row;
                valid = p < out_px;
                sx = tile * 128, sy = 0;
            }
#pragma unroll 1
            for (int cc = 0; cc < C::kNP; cc += kChunk) {
                uint32_t v[C::kG][32];
#pragma unroll
                for (int g = 0; g < C::kG; ++g) {
                    const uint32_t t = tmem + lane_addr + buf * 256 + g * C::kNP + cc;
                    if constexpr (kChunk == 32) tmem_ld32(t, v[g]);
                    else tmem_ld16(t, *reinterpret_cast<uint32_t(*)[16]>(&v[g][0]));
                }
                tmem_ld_wait();
                if constexpr (KIND != C_ENC2 && KIND != C_ENC3) {
                    // two channels per step: h(acc + bias) as one f32x2 add and one f16x2
                    // conversion (each element rounded as alone), then the ReLU (`if (v < 0) v = 0`:
                    // -0 and NaN stay) as a half2 mask
                    const bool relu = KIND == C_ENC_IC || KIND == C_OUT12 ? a.relu == 1 : true;
#pragma unroll
                    for (int j = 0; j < kChunk; j += 2) {
                        const int c = cc + j;
                        if (c >= C::kN) break;  // (kN is even)
                        const float2 b = *reinterpret_cast<const float2*>(&bars->bias[c]);
                        float s0, s1;
                        f2_unpack(f2_add(f2_pack(__uint_as_float(v[0][j]), __uint_as_float(v[0][j + 1])),
                                         f2_pack(b.x, b.y)),
                                  s0, s1);
                        uint32_t h = pack_h2(s0, s1);
                        if (relu) {
                            const __half2 hv = *reinterpret_cast<const __half2*>(&h);
                            h &= ~__hlt2_mask(hv, __float2half2_rn(0.0f));
                        }
                        if (tma_out) {
                            ob[c * 128 + row] = (unsigned short)(h & 0xffffu);
                            ob[(c + 1) * 128 + row] = (unsigned short)(h >> 16);
                        } else if (valid) {
                            a.out[(size_t)c * out_px + p] = __ushort_as_half((unsigned short)(h & 0xffffu));
                            a.out[(size_t)(c + 1) * out_px + p] = __ushort_as_half((unsigned short)(h >> 16));
                        }
                    }
                    continue;
                }
#pragma unroll
                for (int j = 0; j < kChunk; ++j) {
                    const int c = cc + j;
                    if (c >= C::kN) break;
                    const float b = bars->bias[c];
                    // one coopVecMatMulAddNV product: h(acc + bias)
                    const uint16_t p0 = h_bits(__fadd_rn(__uint_as_float(v[0][j]), b));
                    uint16_t o;
                    if constexpr (KIND == C_ENC2) {
                        // strided_conv_split_64ch.comp.glsl:87-91: fp32 (p0 + p1) - b, ReLU, fp16
                        const float p1 = bits_h(h_bits(__fadd_rn(__uint_as_float(v[C::kG - 1][j]), b)));
                        const float s2 = __fsub_rn(__fadd_rn(bits_h(p0), p1), b);
                        o = h_bits(s2 < 0.0f ? 0.0f : s2);
                    } else if constexpr (KIND == C_ENC3) {
                        // strided_conv_split_128ch.comp.glsl:81-86: fp16 running sum, bias removed
                        // per group, then ReLU
                        uint16_t acc = p0;
#pragma unroll
                        for (int g = 1; g < C::kG; ++g) {
                            const float pg = bits_h(h_bits(__fadd_rn(__uint_as_float(v[g][j]), b)));
                            acc = h_bits(__fsub_rn(__fadd_rn(bits_h(acc), pg), b));
                        }
                        o = relu_bits(acc);
                    } else {
                        o = p0;  // (the other kinds take the paired path above)
                    }
                    if (tma_out)
                        ob[c * 128 + row] = o;
                    else if (valid)
                        a.out[(size_t)c * out_px + p] = __ushort_as_half(o);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->acc_empty[buf]);
            if (tma_out) {
                fence_async_shared();  // the tile's stores, for the TMA engine
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->out_full[ob_i]);
                if (warp == store_warp) {  // the issuing warp waits for all four (warp-uniform result)
                    if (!mbar_wait_w(&bars->out_full[ob_i], ob_use & 1, abort)) break;
                    if (issuer) {
                        tma_store_3d(&tm_out, smem_u32(ob), sx, sy, 0);
                        tma_store_commit();
                    }
                }
            }
        }
        if (tma_out && issuer) tma_store_wait0();  // the output is written before the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    if (bars->abort) {
        if (threadIdx.x == 0) atomicOr(a.err, ERR_TIMEOUT);
        const uint64_t t0 = globaltimer();  // let any copy still in flight land
        while (globaltimer() - t0 < 1000000ull) {
        }
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// [G][NP][KGP] K-major fp16 weights (zero padding) from the blob at any alignment, for the weight
// matrices streamed by TMA (over 64 KB).  It waits for the previous kernel before writing: a pass
// of the same kind may still be reading the scratch.
template <int KIND>
__global__ void codec_repack_kernel(const __half* blob, int wo, __half* w) {
    using C = CodecCfg<KIND>;
    grid_dep_wait();
    const int total = C::kG * C::kNP * C::kKGP;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int k = i % C::kKGP, n = (i / C::kKGP) % C::kNP, g = i / (C::kKGP * C::kNP);
        int src = -1;  // element of the group's row in the blob's (channel, tap) order
        if (C::kType == 0) {
            const int t = k / C::kCgP, c = k % C::kCgP;
            if (t < 9 && c < C::kCg) src = c * 9 + t;
        } else if (k < C::kKG) {
            src = k;
        }
        w[i] = n < C::kN && src >= 0 ? blob[wo + (size_t)n * C::kLd + g * C::kKsrc + src] : __float2half(0.0f);
    }
}

// pixelshuffle_sigmoid.comp.glsl:26-56: display pixel (ox, oy) of colour c takes channel
// c*s*s + (oy%s)*s + ox%s of render pixel (ox/s, oy/s), through 1/(1 + exp(-v)) in fp32
// One thread per display pixel (blockIdx.y = display row), its three colours.
__global__ void pixelshuffle_kernel(const __half* in, __half* rgb, int rw, int rh, int dw, int dh, int sc) {
    grid_dep_wait();  // the input is the previous pass's output
    const int ox = blockIdx.x * blockDim.x + threadIdx.x, oy = blockIdx.y;
    if (ox >= dw) return;
    const int64_t rpx = (int64_t)rw * rh, dpx = (int64_t)dw * dh;
    const int64_t at = (int64_t)(oy / sc) * rw + ox / sc;
    const int sub = (oy % sc) * sc + ox % sc;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const float v = __half2float(in[(int64_t)(c * sc * sc + sub) * rpx + at]);
        rgb[c * dpx + (int64_t)oy * dw + ox] = __float2half_rn(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v))));
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
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

// Per-context scratch of the codec passes: the repacked weights of each kind whose matrix is
// streamed (so passes of different kinds never share them).
struct CodecScratch {
    std::mutex mu;
    __half* w[C_COUNT] = {};
};

template <int KIND>
int run_codec(prism_ctx* ctx, const int32_t* q, const __half* weights, size_t weight_elems, __half* feat,
              size_t feat_elems, cudaStream_t s) {
    using C = CodecCfg<KIND>;
    // push constants in each shader's order (the channel counts are fixed by the shaders, which
    // do not read them)
    int in_w, in_h, out_w, out_h, wo, bo, in_off, skip_off = 0, out_off, relu = 1;
    if (KIND == C_ENC_IC || KIND == C_OUT12) {  // {in_ch, out_ch, w, h, w, b, in, out, relu}
        in_w = out_w = q[2];
        in_h = out_h = q[3];
        wo = q[4], bo = q[5], in_off = q[6], out_off = q[7], relu = q[8];
    } else if (C::kType == 0) {  // {in_ch, out_ch, in_w, in_h, out_w, out_h, w, b, in, out}
        in_w = q[2], in_h = q[3], out_w = q[4], out_h = q[5], wo = q[6], bo = q[7], in_off = q[8], out_off = q[9];
    } else {  // {out_w, out_h, in_w, in_h, [up_ch,] skip_ch, w, b, in, skip, out}
        const int* r = KIND == C_DEC3 ? q + 5 : q + 6;
        out_w = q[0], out_h = q[1], in_w = q[2], in_h = q[3];
        wo = r[0], bo = r[1], in_off = r[2], skip_off = r[3], out_off = r[4];
    }
    if (in_w <= 0 || in_h <= 0 || out_w <= 0 || out_h <= 0)
        return set_error(PRISM_E_ARG, "prism_codec_pass: map sizes %dx%d -> %dx%d", in_w, in_h, out_w, out_h);
    const int64_t in_px = (int64_t)in_w * in_h, out_px = (int64_t)out_w * out_h;
    if (out_px > (1ll << 30) || in_px > (1ll << 30)) return set_error(PRISM_E_RANGE, "prism_codec_pass: map too large");
    const int64_t in_ch = C::kType == 1 ? C::kUp : C::kIn;
    if (!in_range(in_off, in_ch * in_px, feat_elems) || !in_range(out_off, (int64_t)C::kN * out_px, feat_elems) ||
        (C::kType == 1 && !in_range(skip_off, (int64_t)C::kSkip * out_px, feat_elems)))
        return set_error(PRISM_E_RANGE, "prism_codec_pass: feature map outside the arena");
    if (!in_range(wo, (int64_t)C::kN * C::kLd, weight_elems) || !in_range(bo, C::kN, weight_elems))
        return set_error(PRISM_E_RANGE, "prism_codec_pass: weights outside the blob");
    auto overlap = [](int64_t a0, int64_t n0, int64_t a1, int64_t n1) { return a0 < a1 + n1 && a1 < a0 + n0; };
    if (overlap(out_off, C::kN * out_px, in_off, in_ch * in_px) ||
        (C::kType == 1 && overlap(out_off, C::kN * out_px, skip_off, C::kSkip * out_px)))
        return set_error(PRISM_E_ARG, "prism_codec_pass: the output map overlaps an input map");
    CUtensorMap tm{};
    if constexpr (!C::kResident) {  // the streamed matrix: repacked into the context's scratch
        if (!ctx->codec) return set_error(PRISM_E_ARG, "prism_codec_pass: context without codec scratch");
        CodecScratch& cs = *static_cast<CodecScratch*>(ctx->codec);
        {
            std::lock_guard<std::mutex> lock(cs.mu);
            if (!cs.w[KIND]) {
                void* w = nullptr;
                if (cudaMalloc(&w, (size_t)C::kG * C::kNP * C::kKGP * 2) != cudaSuccess) {
                    cudaGetLastError();
                    return set_error(PRISM_E_NOMEM, "prism_codec_pass: weight scratch");
                }
                cs.w[KIND] = static_cast<__half*>(w);
            }
        }
        auto fn = encode_tiled();
        if (!fn) return set_error(PRISM_E_CUDA, "cuTensorMapEncodeTiled is not available");
        cuuint64_t dims[2] = {(cuuint64_t)C::kKGP, (cuuint64_t)C::kG * C::kNP};
        cuuint64_t strides[1] = {(cuuint64_t)C::kKGP * 2};
        cuuint32_t box[2] = {64, (cuuint32_t)C::kNP};
        cuuint32_t estr[2] = {1, 1};
        if (fn(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, cs.w[KIND], dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return set_error(PRISM_E_CUDA, "prism_codec_pass: weight tensor map");
        const cudaError_t e = launch_pdl(codec_repack_kernel<KIND>, dim3(64), dim3(256), 0, s, weights, wo, cs.w[KIND]);
        if (e != cudaSuccess) return set_error(PRISM_E_CUDA, "prism_codec_pass: %s", cudaGetErrorString(e));
    }
    CodecArgs a;
    a.in = feat + in_off;
    a.skip = feat + skip_off;
    a.out = feat + out_off;
    a.in_w = in_w, a.in_h = in_h, a.out_w = out_w, a.out_h = out_h;
    a.relu = relu;
    a.blob = weights;
    a.wo = wo;
    a.bo = bo;
    a.err = ctx->err;
    // TMA maps (3-D {x, y, channel}, no swizzle) need 16-byte aligned bases and row pitches: the
    // staged form's input maps, and the output map (else the epilogue stores directly)
    auto fn = encode_tiled();
    auto map3 = [&](CUtensorMap* m, const __half* base, int64_t w, int64_t h, int c, int bw, int bh,
                    CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE) {
        if (!fn || ((uintptr_t)base & 15) || (w * 2) % 16) return false;
        cuuint64_t dims[3] = {(cuuint64_t)w, (cuuint64_t)h, (cuuint64_t)c};
        cuuint64_t strides[2] = {(cuuint64_t)w * 2, (cuuint64_t)(w * h * 2)};
        cuuint32_t box[3] = {(cuuint32_t)bw, (cuuint32_t)bh, (cuuint32_t)c};
        cuuint32_t estr[3] = {1, 1, 1};
        return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    constexpr CUtensorMapSwizzle kSw128 = CU_TENSOR_MAP_SWIZZLE_128B;
    CUtensorMap tin{}, tskip{}, tout{};
    bool staged = false;
    if constexpr (C::kCanStage) {
        if (C::kType == 0)
            staged = map3(&tin, a.in, in_w, in_h, C::kIn, 144, 3);
        else if (C::kType == 1)  // (the staged gather reads up pixel x / 2 unclamped: out_w <= 2 in_w)
            staged = out_w <= 2 * in_w && map3(&tin, a.in, in_w, in_h, C::kUp, 64, 1, kSw128) &&
                     map3(&tskip, a.skip, out_w, out_h, C::kSkip, 64, 1, kSw128);
        else
            staged = map3(&tin, a.in, in_w, in_h, C::kIn, 64, 1, kSw128);
    }
    // output tiles: 128 pixels of one row (staged) or 128 consecutive pixels of the map
    if (staged)
        a.tma_out = CodecCfg<KIND, C::kCanStage>::kEpiGroups == 2 && map3(&tout, a.out, out_w, out_h, C::kN, 128, 1);
    else
        a.tma_out = CodecCfg<KIND, false>::kEpiGroups == 2 && map3(&tout, a.out, out_px, 1, C::kN, 128, 1);
    cudaError_t e;
    if (staged) {
        constexpr bool kStg = C::kCanStage;  // (always true here; keeps the template well-formed)
        const int n_tiles = out_h * ((out_w + 127) / 128);
        constexpr int smem = codec_smem<KIND, kStg>();
        static_assert(smem <= 232448, "shared memory budget");
        e = cudaFuncSetAttribute(codec_tc_kernel<KIND, kStg>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e == cudaSuccess)
            e = launch_pdl(codec_tc_kernel<KIND, kStg>, dim3(std::min(ctx->sm_count, n_tiles)),
                           dim3(CodecCfg<KIND, kStg>::kThreads), smem, s, a, tm, tin, tskip, tout);
    } else {
        const int n_tiles = (int)((out_px + 127) / 128);
        constexpr int smem = codec_smem<KIND, false>();
        static_assert(smem <= 232448, "shared memory budget");
        e = cudaFuncSetAttribute(codec_tc_kernel<KIND, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e == cudaSuccess)
            e = launch_pdl(codec_tc_kernel<KIND, false>, dim3(std::min(ctx->sm_count, n_tiles)),
                           dim3(CodecCfg<KIND, false>::kThreads), smem, s, a, tm, tin, tskip, tout);
    }
    if (e != cudaSuccess) return set_error(PRISM_E_CUDA, "prism_codec_pass: %s", cudaGetErrorString(e));
    return PRISM_OK;
}

}  // namespace

void* codec_scratch_new() { return new CodecScratch; }

void codec_scratch_free(void* p) {
    auto* cs = static_cast<CodecScratch*>(p);
    if (!cs) return;
    for (int k = 0; k < C_COUNT; ++k) cudaFree(cs->w[k]);
    delete cs;
}

}  // namespace prism

using namespace prism;

extern "C" int prism_codec_pass(prism_ctx* ctx, int kind, const int32_t* push, int n_push, const void* weights,
                                size_t weight_elems, void* features, size_t feature_elems, void* rgb,
                                size_t rgb_elems, void* stream) {
    static const int kPush[C_COUNT] = {9, 10, 10, 10, 10, 11, 11, 9, 7};
    if (!ctx || !push || !features) return set_error(PRISM_E_ARG, "prism_codec_pass: NULL argument");
    if (kind < 0 || kind >= C_COUNT) return set_error(PRISM_E_ARG, "prism_codec_pass: kind %d", kind);
    if (n_push != kPush[kind])
        return set_error(PRISM_E_ARG, "prism_codec_pass: kind %d takes %d push constants, got %d", kind, kPush[kind],
                         n_push);
    if (kind != C_PS && !weights) return set_error(PRISM_E_ARG, "prism_codec_pass: NULL weights");
    DeviceGuard g(ctx->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const __half* w = static_cast<const __half*>(weights);
    __half* f = static_cast<__half*>(features);
    switch (kind) {
        case C_ENC_IC: return run_codec<C_ENC_IC>(ctx, push, w, weight_elems, f, feature_elems, s);
        case C_ENC1: return run_codec<C_ENC1>(ctx, push, w, weight_elems, f, feature_elems, s);
        case C_ENC2: return run_codec<C_ENC2>(ctx, push, w, weight_elems, f, feature_elems, s);
        case C_ENC3: return run_codec<C_ENC3>(ctx, push, w, weight_elems, f, feature_elems, s);
        case C_DEC3: return run_codec<C_DEC3>(ctx, push, w, weight_elems, f, feature_elems, s);
        case C_DEC2: return run_codec<C_DEC2>(ctx, push, w, weight_elems, f, feature_elems, s);
        case C_DEC1: return run_codec<C_DEC1>(ctx, push, w, weight_elems, f, feature_elems, s);
        case C_OUT12: return run_codec<C_OUT12>(ctx, push, w, weight_elems, f, feature_elems, s);
        default: break;
    }
    // pixelshuffle_sigmoid {render_w, render_h, display_w, display_h, scale, in_off, out_off}: the RGB
    // output goes to binding 2 (rgb, fp16)
    const int rw = push[0], rh = push[1], dw = push[2], dh = push[3], sc = push[4], in_off = push[5],
              out_off = push[6];
    if (!rgb) return set_error(PRISM_E_ARG, "prism_codec_pass: NULL rgb buffer");
    if (rw <= 0 || rh <= 0 || dw <= 0 || dh <= 0 || sc < 1 || (int64_t)dw > (int64_t)rw * sc ||
        (int64_t)dh > (int64_t)rh * sc)
        return set_error(PRISM_E_ARG, "prism_codec_pass: pixel shuffle %dx%d x%d -> %dx%d", rw, rh, sc, dw, dh);
    if (!in_range(in_off, (int64_t)3 * sc * sc * rw * rh, feature_elems) ||
        !in_range(out_off, (int64_t)3 * dw * dh, rgb_elems))
        return set_error(PRISM_E_RANGE, "prism_codec_pass: pixel shuffle outside its buffers");
    if (dh > 65535) return set_error(PRISM_E_RANGE, "prism_codec_pass: display height %d", dh);
    cudaError_t e = launch_pdl(pixelshuffle_kernel, dim3((dw + 255) / 256, dh), dim3(256), 0, s,
                               static_cast<const __half*>(f + in_off), static_cast<__half*>(rgb) + out_off, rw, rh, dw,
                               dh, sc);
    if (e != cudaSuccess) return set_error(PRISM_E_CUDA, "prism_codec_pass: %s", cudaGetErrorString(e));
    return PRISM_OK;
}

extern "C" int prism_ctx_status(prism_ctx* ctx, void* stream) {
    if (!ctx) return set_error(PRISM_E_ARG, "prism_ctx_status: NULL");
    DeviceGuard g(ctx->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint32_t e = 0;
    if (cudaMemcpyAsync(&e, ctx->err, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemsetAsync(ctx->err, 0, 4, s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
        return set_error(PRISM_E_CUDA, "prism_ctx_status: %s", cudaGetErrorString(cudaGetLastError()));
    if (e & ERR_TIMEOUT) return set_error(PRISM_E_TIMEOUT, "a device-side wait timed out (error word 0x%x)", e);
    return PRISM_OK;
}
