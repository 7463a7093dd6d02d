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
// Each runs here as an implicit GEMM: a tile is 128 consecutive output pixels (rows = MMA M),
// N = output channels, K = the shader's input vector (channel, ky, kx order), one TMEM
// accumulator per channel group.  Feature maps are CHW fp16 at element offsets of the caller's
// arena, read with plain loads at any alignment; the weights are repacked by a small kernel into
// an aligned K-major copy ([group][N][K padded to 64]) that the weight ring loads by TMA.
// The ninth shader, pixelshuffle_sigmoid, is elementwise (SIMT kernel at the end of the file).
//
// Warp roles (448 threads):
//   warp 0      producer: weight K-blocks {64 K, N rows} by TMA (128B swizzle, no multicast)
//   warp 1      TMEM owner + tcgen05.mma issuer
//   warps 2-9   gather: warp 2 + 4h + q fills rows 32q.. with K columns [32h, 32h + 32) of every
//               K-block (the patch values, zero outside the map), 16-byte stores into the
//               swizzled A tile
//   warps 10-13 epilogue: TMEM -> the shader's rounding / group rule -> CHW stores (each warp
//               instruction writes 32 consecutive pixels of one channel)
// Weight matrices of up to 64 KB (all but the two split convolutions) are loaded into shared
// memory once per CTA and an 8-stage ring carries the A K-blocks; the split convolutions' weights
// stream through a 4-stage ring of {A K-block 16 KB, B K-block N x 128 B}.  Every wait is
// bounded (common.cuh); on timeout the CTA sets the context's error word and winds down.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "host_util.h"

namespace prism {
namespace {

// kinds in the order of prism_codec_kind (include/prism_moe.h)
enum : int { C_ENC_IC = 0, C_ENC1, C_ENC2, C_ENC3, C_DEC3, C_DEC2, C_DEC1, C_OUT12, C_PS, C_COUNT };

template <int KIND>
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
    static constexpr int kStages = kResident ? 8 : 4;
    static constexpr int kStageBytes = kResident ? 16384 : 32768;  // A (+ B when streamed)
    static constexpr int kWOff = kStages * kStageBytes;         // resident weights
    static constexpr int kBarOff = kWOff + (kResident ? (kWBytes + 1023) / 1024 * 1024 : 0);
};

constexpr int kThreads = 32 * 14;
constexpr int kMaxStages = 8;
constexpr int kABytes = 128 * 128;  // one A K-block: 128 rows x 64 fp16, SW128

struct CodecArgs {
    const __half* in;    // conv / pw: the input map; dec: the deeper map (CHW)
    const __half* skip;  // dec: the skip map at the output resolution (CHW)
    __half* out;         // the output map (CHW)
    int in_w, in_h, out_w, out_h;
    int relu;            // conv3x3_9ch / pw: the push constant (1 = ReLU)
    const __half* blob;  // the weights arena: matrix at element wo, biases at bo (any alignment)
    int wo, bo;
    uint32_t* err;
};

struct Bars {
    uint64_t a_full[kMaxStages], b_full[kMaxStages], empty[kMaxStages];
    uint64_t acc_full[2], acc_empty[2], drain;
    uint32_t tmem_base;
    int abort;
    float bias[128];
};
template <int KIND>
constexpr int codec_smem() {  // + alignment slack of the dynamic base
    return CodecCfg<KIND>::kBarOff + (int)sizeof(Bars) + 1024;
}

PRISM_DEV uint16_t h_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }
PRISM_DEV float bits_h(uint16_t b) { return __half2float(__ushort_as_half(b)); }
// `if (v < 0) v = 0` on an fp16 value (negative zero stays, as in the shaders)
PRISM_DEV uint16_t relu_bits(uint16_t b) { return bits_h(b) < 0.0f ? (uint16_t)0 : b; }

template <int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    codec_tc_kernel(const CodecArgs a, const __grid_constant__ CUtensorMap tm_w) {
    using C = CodecCfg<KIND>;
    constexpr int kStages = C::kStages, kStageBytes = C::kStageBytes;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    Bars* bars = reinterpret_cast<Bars*>(smem + C::kBarOff);
    volatile int* abort = &bars->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int out_px = a.out_w * a.out_h;
    const int n_tiles = (out_px + 127) >> 7;

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
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        constexpr int kChunk = C::kNP >= 32 && C::kG == 1 ? 32 : 16;  // columns per TMEM load and group
        uint32_t it = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
            const int buf = C::kAccBufs == 2 ? (int)(it & 1) : 0;
            const uint32_t use = C::kAccBufs == 2 ? (it >> 1) : it;
            if (!mbar_wait(&bars->acc_full[buf], use & 1, abort)) break;
            tc_fence_after();
            const int p = tile * 128 + row;
            const bool valid = p < out_px;
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
                    } else if constexpr (KIND == C_ENC_IC || KIND == C_OUT12) {
                        o = a.relu == 1 ? relu_bits(p0) : p0;
                    } else {
                        o = relu_bits(p0);
                    }
                    if (valid) a.out[(size_t)c * out_px + p] = __ushort_as_half(o);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->acc_empty[buf]);
        }
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
    const int n_tiles = (int)((out_px + 127) / 128);
    constexpr int smem = codec_smem<KIND>();
    static_assert(smem <= 232448, "shared memory budget");
    cudaError_t e = cudaFuncSetAttribute(codec_tc_kernel<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) {
        e = launch_pdl(codec_tc_kernel<KIND>, dim3(std::min(ctx->sm_count, n_tiles)), dim3(kThreads), smem, s, a, tm);
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
