// attn_tc.cu - fused windowed-attention block on the sm_100a tensor cores.
//
// Computes, for every 8x8 window of every frame, the first pass of a Prism MoE block
// (split2_qkv_attn_d256.comp.glsl:24-79) and the router that follows it
// (moe_router.comp.glsl:24-52 with N-wide logits, moe_ffn_16exp.comp.glsl:27-34), or the
// attention half of a dense block (attention_windowed_d256.comp.glsl:54-141 at D = 256,
// attention_windowed.comp.glsl:53-148 at D = 128, no router):
//     y = x + Wo . MHA_window(x) + bo            (fp16, masked store of valid tokens)
//     assign[t] = argmax_e (Wr . y + br)[e]      (first maximum), counts[e] += 1
//
// One persistent CTA per SM walks tiles of two windows (128 rows; row = window slot
// li = 8*ty + tx, slots outside the frame are the reference's phantom zero tokens:
// the 4-D TMA load zero-fills them and they take part as keys, :31-37, :60).
// Per tile and head h (D/32 heads x 32; the text below is for D = 256):
//   QKV_h   TMEM[96]  = X[128x256] . Wqkv_h^T        (tcgen05, K = 256)
//   drain   Q_h, K_h (fp16, K-major SW64) and V_h (fp16, key-major SW64: the MN-major B
//           operand of PV, so it is stored like K, no transpose) to smem
//   S_h     TMEM[128] = Q_h . K_h^T                   (both windows; rows use their own)
//   softmax fp32 per row over its window's 64 keys (scale, max, exp, sum as :60-66),
//           P = fp16(exp(s - max)) written over S in TMEM (tcgen05.st), the other
//           window's keys zero
//   PV_h    TMEM[32]  = P[128x128] (A from TMEM) . V_h  (block-diagonal P)
//   O_h     = fp16(PV * 1/max(sum, 1e-6))  -> attention-output tile (head pair)
//   PO     += O_pair[128x64] . Wo[:, pair]^T          (TMEM[256], K split by head pair)
// then y = fp16(fp16(PO + bo) + x) overwrites X in smem, is stored with a 4-D TMA
// store (rows outside the frame are clipped = the masked store :78), and the router
// GEMM TMEM = y . Wr^T gives the logits for the argmax.
//
// Warp roles (320 threads):
//   warp 0      TMA producer: X tile (4-D window boxes), weight ring (QKV_h, Wo, Wr)
//   warp 1      TMEM owner + tcgen05.mma issuer
//   warps 2-5   softmax group: S_h -> P_h, O_h -> attention-output tile, y columns 128..255
//   warps 6-9   drain group: QKV_h -> Q/K/V smem, y columns 0..127, store, router
// Thread = tile row = TMEM lane in both groups (warp w reads lanes 32*(w%4)..).
// The two groups run one head apart and the MMA warp issues QKV_{h+1} right after S_h.
// Weights stream through a 2 x 48 KB ring in whole operands, one TMA load each: a
// head's Wqkv rows at full K (K-block-major copy, 3-D map), a head pair's Wo columns,
// up to 96 router rows.  On B200 every load costs the producer/consumer hand-off
// (~300-400 cycles) whatever its size, so few large loads keep the stream ahead.
// Every wait is bounded (common.cuh); on timeout the CTA sets the error word and
// winds down.  No TMA multicast.
#include "attn_parts.cuh"
#include "attn_tc.cuh"
#include "common.cuh"

namespace prism {
namespace {

constexpr int kThreads = 320;  // 10 warps
constexpr int kStages = 2;
constexpr int kRouterRows = 96;  // router rows per ring stage

// Shapes of the kernel for model width D (256: the MoE / "Standard" blocks, 128: the
// "Baseline" block, attention_windowed.comp.glsl): D / 64 K-blocks, D / 32 heads of 32.
template <int D>
struct AttnCfg {
    static_assert(D == 128 || D == 256, "model width");
    static constexpr int kKB = D / 64;      // 64-wide K-blocks of X, y and the weights
    static constexpr int kHeads = D / 32;
    // weight ring stage: a head's Wqkv rows at full K ([96][128 B] per K-block) or a pair's
    // Wo columns ([D][128 B]); router rows at D = 256 (96 x 4 K-blocks)
    static constexpr int kStage = 96 * 128 * kKB > D * 128 ? 96 * 128 * kKB : D * 128;
    // shared-memory map (offsets from the 1024-aligned base)
    static constexpr int kOffX = 0;                    // kKB K-blocks x [128][128 B]; y overwrites it
    static constexpr int kOffQ = kOffX + 16384 * kKB;  // Q_h [128][64 B] SW64 8 KB
    static constexpr int kOffK = kOffQ + 8192;         // K_h [128][64 B] SW64 8 KB
    static constexpr int kOffV = kOffK + 8192;         // V_h, 2 buffers (head parity) x [128 keys][64 B] SW64
    static constexpr int kOffAO = kOffV + 16384;       // [128][128 B] SW128 16 KB (one head pair)
    static constexpr int kOffW = kOffAO + 16384;       // weight ring
    static constexpr int kOffBar = kOffW + kStages * kStage;
};

// Head pair whose out-projection the MMA warp issues at head h of `heads`: pair p = (2p, 2p + 1)
// at head 2p + 2 (behind QKV_{2p+3}), the last pair after the last PV; -1 at the other heads.
PRISM_DEV constexpr int po_pair(int h, int heads) {
    return h == heads - 1 ? heads / 2 - 1 : (h >= 2 && (h & 1) == 0) ? h / 2 - 1 : -1;
}

// TMEM columns
constexpr uint32_t kTPO = 0;     // out-projection accumulator [256]; router logits reuse [0, npad)
constexpr uint32_t kTQKV = 256;  // QKV_h [96]
constexpr uint32_t kTS = 352;    // S_h [128] fp32; P_h overwrites [352, 416) as fp16 pairs
constexpr uint32_t kTO = 480;    // PV_h [32]

struct Bars {
    float bqkv[768];  // biases staged once per CTA (read as warp-uniform broadcasts)
    float bo[256];
    float br[256];
    uint64_t full[kStages], empty[kStages];
    uint64_t x_full[4], x_free[4], qkv_full, qkv_drained, s_full, p_ready, o_full, o_drained;
    uint64_t ao_ready, ao_free, po_full, po_drained, y_ready[4], lg_full, lg_drained, drain, ep_done;
    uint32_t tmem_base;
    int abort;
    int hist[256];
};
template <int D>
constexpr int attn_smem() {  // + alignment slack of the dynamic base
    return AttnCfg<D>::kOffBar + (int)sizeof(Bars) + 1024;
}
static_assert(attn_smem<256>() <= 232448 && attn_smem<128>() <= 232448, "shared memory budget");

struct Counter {  // phase bookkeeping of one barrier as seen by one role
    uint32_t n = 0;
    PRISM_DEV uint32_t next() { return (n++) & 1u; }              // consumer: wait phase parity
    PRISM_DEV uint32_t next_free() { return ((n++) & 1u) ^ 1u; }  // producer of a free slot
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const AttnTcArgs a, const __grid_constant__ CUtensorMap tm_x,
                   const __grid_constant__ CUtensorMap tm_y, const __grid_constant__ CUtensorMap tm_wqkv,
                   const __grid_constant__ CUtensorMap tm_wo, const __grid_constant__ CUtensorMap tm_wr) {
    using Cfg = AttnCfg<D>;
    constexpr int kKB = Cfg::kKB, kHeads = Cfg::kHeads, kStage = Cfg::kStage;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = smem_align1k(smem_raw);
    unsigned char* sX = smem + Cfg::kOffX;
    unsigned char* sQ = smem + Cfg::kOffQ;
    unsigned char* sK = smem + Cfg::kOffK;
    unsigned char* sV = smem + Cfg::kOffV;  // buffer b at +8192*b
    unsigned char* sAO = smem + Cfg::kOffAO;
    unsigned char* sW = smem + Cfg::kOffW;
    Bars* bars = reinterpret_cast<Bars*>(smem + Cfg::kOffBar);
    volatile int* abort = &bars->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wx_n = (a.W + 7) >> 3, wy_n = (a.H + 7) >> 3;
    const int win_per_frame = wx_n * wy_n;
    const int n_windows = win_per_frame * a.frames;
    const int n_tiles = (n_windows + 1) >> 1;
    const bool router = D == 256 && a.n_experts > 0;  // MoE blocks are dim 256
    const int npad = a.n_experts_pad;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int kb = 0; kb < kKB; ++kb) {  // the X tile moves K-block by K-block at tile ends
            mbar_init(&bars->x_full[kb], 1);
            mbar_init(&bars->x_free[kb], 1);   // y K-block read by the router GEMM (commit)
            mbar_init(&bars->y_ready[kb], 8);  // y K-block written (both SIMT groups, a chunk each)
        }
        mbar_init(&bars->qkv_full, 1);
        mbar_init(&bars->qkv_drained, 4);
        mbar_init(&bars->s_full, 1);
        mbar_init(&bars->p_ready, 4);
        mbar_init(&bars->o_full, 1);
        mbar_init(&bars->o_drained, 4);
        mbar_init(&bars->ao_ready, 4);
        mbar_init(&bars->ao_free, 1);
        mbar_init(&bars->po_full, 1);
        mbar_init(&bars->po_drained, 8);  // both SIMT groups write y
        mbar_init(&bars->lg_full, 1);
        mbar_init(&bars->lg_drained, 4);
        mbar_init(&bars->drain, 1);
        mbar_init(&bars->ep_done, 4);
        bars->abort = 0;
        fence_barrier_init();
        fence_async_shared();
    }
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        bars->hist[i] = 0;
        bars->bo[i] = i < D ? a.bo[i] : 0.0f;
        bars->br[i] = router && i < a.n_experts ? a.br[i] : 0.0f;
    }
    for (int i = threadIdx.x; i < 3 * D; i += blockDim.x) bars->bqkv[i] = a.bqkv[i];
    if (warp == 1) tmem_alloc(&bars->tmem_base, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    // Programmatic dependent launch: the next kernel may place its CTAs now (they wait for this
    // grid to complete before reading its results).  This grid's own wait for the previous
    // kernels is taken only by the roles that touch their memory: the producer after the first
    // weight load (x, and y over the previous kernel's input) and the drain group (routing
    // outputs); the weights and biases are never written by a forward.
    grid_dep_launch();

    if (warp == 0) {
        // ============================ TMA producer ============================
        if (lane == 0) {
            prefetch_tmap(&tm_x);
            prefetch_tmap(&tm_wqkv);
            prefetch_tmap(&tm_wo);
            if (router) prefetch_tmap(&tm_wr);
            int stage = 0;
            uint32_t phase = 0;
            Counter c_xfree[4];
            bool ok = true;
            // one ring stage = one TMA load (3-D maps: rows c1.. at every K-block)
            auto ring_load = [&](const CUtensorMap* map, bool kb3d, int c0, int c1, uint32_t bytes) -> bool {
                if (!mbar_wait(&bars->empty[stage], phase ^ 1, abort)) return false;
                mbar_expect_tx(&bars->full[stage], bytes);
                if (kb3d)
                    tma_load_3d(smem_u32(sW + stage * kStage), map, &bars->full[stage], 0, c1, 0);
                else
                    tma_load_2d(smem_u32(sW + stage * kStage), map, &bars->full[stage], c0, c1);
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1;
                }
                return true;
            };
            const int r_rows = npad < kRouterRows ? npad : kRouterRows;  // rows per router load
            // y of the previous tile: the TMA store of K-block kb as soon as both groups wrote it
            int prev = -1;  // previous tile
            Counter c_yst[4];
            auto store_y = [&](int t) {
                for (int kb = 0; kb < kKB; ++kb) {
                    if (!mbar_wait(&bars->y_ready[kb], c_yst[kb].next(), abort)) return false;
                    for (int half = 0; half < 2; ++half) {
                        const int w = 2 * t + half;
                        if (w >= n_windows) continue;
                        const int f = w / win_per_frame, wl = w % win_per_frame;
                        tma_store_4d(&tm_y, smem_u32(sX + kb * 16384 + half * 8192), kb * 64, (wl % wx_n) * 8,
                                     (wl / wx_n) * 8, f);
                    }
                    tma_store_commit();
                }
                return true;
            };
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                int wf[2], wxx[2], wyy[2];
                for (int half = 0; half < 2; ++half) {
                    const int w = 2 * tile + half;
                    // a missing second window loads an out-of-range frame: zero fill
                    wf[half] = w < n_windows ? w / win_per_frame : a.frames;
                    const int wl = w < n_windows ? w % win_per_frame : 0;
                    wyy[half] = wl / wx_n;
                    wxx[half] = wl % wx_n;
                }
                // same order as the MMA warp consumes: QKV_0 (its stage frees when the previous
                // tile's last out-projection completes), then per head h QKV_{h+1} and, at heads
                // 2, 4, 6 and after head 7, the Wo columns of the pair before
                constexpr uint32_t kQkvBytes = 96 * 128 * kKB, kWoBytes = D * 128;
                ok = ring_load(&tm_wqkv, true, 0, 0, kQkvBytes);
                if (prev < 0) grid_dep_wait();
                if (ok && prev >= 0) ok = store_y(prev);
                // each X K-block once the previous tile's y K-block has been read by its store
                // and by the router GEMM (x_free)
                for (int kb = 0; kb < kKB && ok; ++kb) {
                    if (prev >= 0) {  // y K-block kb has been read out by its store
                        if (kKB - 1 - kb == 3) tma_store_wait_read<3>();
                        else if (kKB - 1 - kb == 2) tma_store_wait_read<2>();
                        else if (kKB - 1 - kb == 1) tma_store_wait_read<1>();
                        else tma_store_wait_read<0>();
                    }
                    if (!mbar_wait(&bars->x_free[kb], c_xfree[kb].next_free(), abort)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&bars->x_full[kb], 16384);
                    for (int half = 0; half < 2; ++half)
                        tma_load_4d(smem_u32(sX + kb * 16384 + half * 8192), &tm_x, &bars->x_full[kb], kb * 64,
                                    wxx[half] * 8, wyy[half] * 8, wf[half]);
                }
                if (!ok) break;
                prev = tile;
                for (int h = 0; h < kHeads && ok; ++h) {
                    if (h < kHeads - 1) ok = ring_load(&tm_wqkv, true, 0, (h + 1) * 96, kQkvBytes);
                    const int p = po_pair(h, kHeads);
                    if (p >= 0 && ok) ok = ring_load(&tm_wo, false, p * 64, 0, kWoBytes);
                }
                if (router)
                    for (int r0 = 0; r0 < npad && ok; r0 += kRouterRows)
                        ok = ring_load(&tm_wr, true, 0, r0, (uint32_t)r_rows * 512);
            }
            if (ok && prev >= 0) store_y(prev);
            tma_store_wait0();
        }
    } else if (warp == 1) {
        // ============================ MMA issuer ==============================
        // Order per tile: QKV_0; for h: [Q,K,V of h drained] S_h, QKV_{h+1}, at h = 2, 4, 6
        // [pair before ready] PO += ..., [P_h ready, O columns free] PV_h; after PV_7 the
        // last pair's PO
        {
            const uint32_t id_qkv = idesc_f16(128, 96), id_s = idesc_f16(128, 128), id_pv = idesc_f16(128, 32) | (1u << 16) /* B = V MN-major */,
                           id_po = idesc_f16(128, D);
            const int r_rows = npad < kRouterRows ? npad : kRouterRows;
            int stage = 0;
            uint32_t phase = 0;
            Counter c_xfull[4], c_qkvd, c_pr, c_od, c_aor, c_pod, c_yr[4], c_lgd;
            bool ok = true;
            bool first_tile = true;
            auto ring_wait = [&]() -> uint32_t {
                if (!mbar_wait_w(&bars->full[stage], phase, abort)) {
                    ok = false;
                    return 0;
                }
                tc_fence_after();
                return smem_u32(sW + stage * kStage);
            };
            auto ring_release = [&]() {
                mma_commit_w(&bars->empty[stage]);
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1;
                }
            };
            auto wait = [&](uint64_t* bar, uint32_t par) {
                if (ok && !mbar_wait_w(bar, par, abort)) ok = false;
                tc_fence_after();
            };
            const uint32_t xs = smem_u32(sX);
            auto issue_qkv = [&](bool first_of_tile) {  // the tile's first: X K-blocks as they land
                const uint32_t b = ring_wait();  // Wqkv_h: K-block kc at +kc * 96 rows
                if (ok) {
#pragma unroll 1
                    for (int kc = 0; kc < kKB; ++kc) {
                        if (first_of_tile) wait(&bars->x_full[kc], c_xfull[kc].next());
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            mma_f16_ss_w(tmem + kTQKV, sdesc(xs + kc * 16384 + k * 32, SW128),
                                         sdesc(b + kc * 12288 + k * 32, SW128), id_qkv, (kc | k) != 0);
                    }
                    ring_release();
                }
                mma_commit_w(&bars->qkv_full);
            };
            // ---- PO += O_pair . Wo[:, pair]^T for the pair po_pair(h): issued behind QKV_{h+1}
            // rather than right after the pair's second PV, so the wait for the pair's
            // attention output and the four N = 256 MMAs stay off the QKV -> S chain
            auto issue_po = [&](int h) {
                const int p = po_pair(h, kHeads);
                if (p < 0) return;
                wait(&bars->ao_ready, c_aor.next());
                if (p == 0 && !first_tile) {  // PO and the previous tile's logits drained
                    wait(&bars->po_drained, c_pod.next());
                    wait(&bars->lg_drained, c_lgd.next());
                }
                const uint32_t b = ring_wait();  // Wo[:, pair]: all D output rows, N = D
                if (ok) {
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        mma_f16_ss_w(tmem + kTPO, sdesc(smem_u32(sAO) + k * 32, SW128), sdesc(b + k * 32, SW128),
                                     id_po, (p > 0) || (k != 0));
                    ring_release();
                }
                mma_commit_w(&bars->ao_free);
            };
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                issue_qkv(true);
                for (int h = 0; h < kHeads && ok; ++h) {
                    const uint32_t vs = smem_u32(sV + (h & 1) * 8192);
                    wait(&bars->qkv_drained, c_qkvd.next());
                    // ---- S_h = Q K^T
                    for (int k = 0; k < 2; ++k)
                        mma_f16_ss_w(tmem + kTS, sdesc(smem_u32(sQ) + k * 32, SW64), sdesc(smem_u32(sK) + k * 32, SW64),
                                   id_s, k != 0);
                    mma_commit_w(&bars->s_full);
                    if (h < kHeads - 1) issue_qkv(false);
                    if (h < kHeads - 1) issue_po(h);
                    wait(&bars->p_ready, c_pr.next());
                    // O columns free once the softmax group drained the previous head
                    if (h > 0 || !first_tile) wait(&bars->o_drained, c_od.next());
                    // ---- O_h = P V, P (fp16) read from TMEM: 16 keys = 8 columns per MMA
                    for (int k = 0; k < 8; ++k)
                        mma_f16_ts_w(tmem + kTO, tmem + kTS + k * 8, sdesc(vs + k * 1024, SW64), id_pv, k != 0);
                    mma_commit_w(&bars->o_full);
                    if (h == kHeads - 1) issue_po(h);
                }
                mma_commit_w(&bars->po_full);
                // ---- router logits = y . Wr^T, K-block by K-block as y lands; each X K-block
                // is released (x_free) after its last router MMA
                if (router) {
                    const uint32_t ys = xs;  // y overwrote X
                    int yw = 0;  // y K-blocks waited for
                    auto need_y = [&](int kb) {
                        for (; yw <= kb && yw < 4; ++yw) wait(&bars->y_ready[yw], c_yr[yw].next());
                    };
                    // up to 96 expert rows per stage (K-block kc at +kc * r_rows rows); their
                    // logits land in PO columns r0 .., whose y K-blocks must have been drained
                    for (int r0 = 0; r0 < npad && ok; r0 += kRouterRows) {
                        const uint32_t b = ring_wait();
                        if (!ok) break;
                        const int n = npad - r0 < r_rows ? npad - r0 : r_rows;
                        const uint32_t id_r = idesc_f16(128, n);
                        const bool last_stage = r0 + kRouterRows >= npad;
                        need_y((r0 + n - 1) >> 6);
#pragma unroll 1
                        for (int kc = 0; kc < 4; ++kc) {
                            need_y(kc);
#pragma unroll
                            for (int k = 0; k < 4; ++k)
                                mma_f16_ss_w(tmem + kTPO + r0, sdesc(ys + kc * 16384 + k * 32, SW128),
                                             sdesc(b + kc * r_rows * 128 + k * 32, SW128), id_r, (kc | k) != 0);
                            if (last_stage) mma_commit_w(&bars->x_free[kc]);
                        }
                        ring_release();
                    }
                } else {
                    for (int kc = 0; kc < kKB; ++kc) {
                        wait(&bars->y_ready[kc], c_yr[kc].next());
                        mma_commit_w(&bars->x_free[kc]);
                    }
                }
                mma_commit_w(&bars->lg_full);
                first_tile = false;
            }
            mma_commit_w(&bars->drain);
            mbar_wait_w(&bars->drain, 0, abort);
        }
    } else if (warp < 6) {
        // ============================ softmax group ===========================
        const int quad = warp & 3;
        const int r = quad * 32 + lane;  // tile row = TMEM lane
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const int wnd = r >> 6;  // which window of the tile
        const float c2 = a.scale * 1.4426950408889634f;  // scale * log2(e)
        const int nkeys = a.n_keys;
        Counter c_s, c_o, c_aof, c_po;
        bool ok = true;
        bool first_pair = true;
        auto wait = [&](uint64_t* bar, uint32_t par) {
            if (ok && !mbar_wait(bar, par, abort)) ok = false;
            tc_fence_after();
        };
        auto arrive = [&](uint64_t* bar) {
            __syncwarp();
            if (lane == 0) mbar_arrive(bar);
        };
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
            for (int h = 0; h < kHeads && ok; ++h) {
                // ---- softmax over this row's window (split2_qkv_attn_d256.comp.glsl:59-66)
                wait(&bars->s_full, c_s.next());
                if (!ok) break;
                uint32_t sv[64];
                tmem_ld32(tmem + lane_addr + kTS + wnd * 64, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
                tmem_ld32(tmem + lane_addr + kTS + wnd * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
                tmem_ld_wait();
                uint32_t pk[32];
                const float se = attn_softmax_row(sv, c2, nkeys, pk);
                const float inv = __frcp_rn(fmaxf(se, 1e-6f));
                attn_store_p(tmem + lane_addr + kTS, wnd, pk);
                tc_fence_before();
                arrive(&bars->p_ready);

                // ---- O_h = PV / sum -> fp16 attention output (head pair tile)
                wait(&bars->o_full, c_o.next());
                if (!ok) break;
                if ((h & 1) == 0 && !first_pair) wait(&bars->ao_free, c_aof.next());
                if (!ok) break;
                {
                    uint32_t v[32];
                    tmem_ld32(tmem + lane_addr + kTO, v);
                    tmem_ld_wait();
                    uint32_t po[16];
                    attn_scale_o(v, inv, po);
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        *reinterpret_cast<uint4*>(sAO + sw128_off(r, (h & 1) * 4 + c)) =
                            make_uint4(po[4 * c], po[4 * c + 1], po[4 * c + 2], po[4 * c + 3]);
                }
                tc_fence_before();
                arrive(&bars->o_drained);
                if (h & 1) {
                    fence_async_shared();
                    arrive(&bars->ao_ready);
                    first_pair = false;
                }
            }
            if (!ok) break;
            // ---- y: the odd 32-column chunk of every K-block
            wait(&bars->po_full, c_po.next());
            if (!ok) break;
            y_share<kKB>(sX, tmem + lane_addr, r, bars->bo, 1, bars->y_ready, lane);
            tc_fence_before();
            arrive(&bars->po_drained);
        }
    } else {
        // ============================ drain group =============================
        const int quad = warp & 3;
        const int r = quad * 32 + lane;  // tile row = TMEM lane
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const int wnd = r >> 6;
        const int li = r & 63;
        const int ty = li >> 3, tx = li & 7;
        Counter c_qkv, c_po, c_lg;
        bool ok = true;
        bool first_tile = true;
        auto wait = [&](uint64_t* bar, uint32_t par) {
            if (ok && !mbar_wait(bar, par, abort)) ok = false;
            tc_fence_after();
        };
        auto arrive = [&](uint64_t* bar) {
            __syncwarp();
            if (lane == 0) mbar_arrive(bar);
        };
        grid_dep_wait();  // the routing outputs of the previous block are consumed
        // QKV_h (TMEM) -> fp16 Q, K (K-major SW64) and V (key-major SW64, buffer h&1)
        auto drain_qkv = [&](int h) {
            wait(&bars->qkv_full, c_qkv.next());
            if (!ok) return;
            attn_drain_row(tmem + lane_addr + kTQKV, bars->bqkv + h * 96, r, sQ, sK, sV + (h & 1) * 8192);
            fence_async_shared();
            tc_fence_before();
            arrive(&bars->qkv_drained);
        };
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
            const int w = 2 * tile + wnd;
            const bool win_ok = w < n_windows;
            const int f = win_ok ? w / win_per_frame : 0;
            const int wl = win_ok ? w % win_per_frame : 0;
            const int wy = wl / wx_n, wx = wl % wx_n;
            const int gy = wy * 8 + ty, gx = wx * 8 + tx;
            const bool valid = win_ok && gy < a.H && gx < a.W;
            const int64_t token = (int64_t)f * a.W * a.H + (int64_t)gy * a.W + gx;
            for (int h = 0; h < kHeads && ok; ++h) drain_qkv(h);
            if (!ok) break;

            // ---- y: the even 32-column chunk of every K-block (the producer stores y)
            wait(&bars->po_full, c_po.next());
            if (!ok) break;
            y_share<kKB>(sX, tmem + lane_addr, r, bars->bo, 0, bars->y_ready, lane);
            tc_fence_before();
            arrive(&bars->po_drained);

            // ---- router: logits (PO columns [0, npad)) = fp16(y . Wr^T + br), first maximum
            wait(&bars->lg_full, c_lg.next());
            if (!ok) break;
            if (router) {
                const float* br = bars->br;
                const int best = router_argmax(tmem + lane_addr + kTPO, npad, a.n_experts, [br](int e) { return br[e]; });
                tc_fence_before();
                arrive(&bars->lg_drained);  // the logits are read: the next tile's out-projection may go
                route_token(a, bars->hist, valid, token, best, lane);
            } else {
                tc_fence_before();
                arrive(&bars->lg_drained);
            }
            first_tile = false;
        }
        // flush the CTA's routing histogram once every drain warp is done
        arrive(&bars->ep_done);
        if (mbar_wait(&bars->ep_done, 0, abort) && router && !a.perm_b)
            for (int e = threadIdx.x - 192; e < a.n_experts; e += 128)
                if (bars->hist[e]) atomicAdd(&a.counts[e], bars->hist[e]);
    }

    tc_fence_before();
    __syncthreads();
    if (bars->abort) {
        if (threadIdx.x == 0) atomicOr(a.err, ERR_TIMEOUT);
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

int attn_tc_smem_bytes(int dim) { return dim == 128 ? attn_smem<128>() : attn_smem<256>(); }

namespace {
template <int D>
cudaError_t launch_attn(const AttnTcArgs& a, const CUtensorMap& x, const CUtensorMap& y, const CUtensorMap& wqkv,
                        const CUtensorMap& wo, const CUtensorMap& wr, int grid, cudaStream_t s) {
    constexpr int smem = attn_smem<D>();
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(attn_tc_kernel<D>, dim3(grid), dim3(kThreads), smem, s, a, x, y, wqkv, wo, wr);
}
}  // namespace

cudaError_t launch_attn_tc(int dim, const AttnTcArgs& a, const CUtensorMap& x, const CUtensorMap& y,
                           const CUtensorMap& wqkv, const CUtensorMap& wo, const CUtensorMap& wr, int grid,
                           cudaStream_t s) {
    if (dim == 128) return launch_attn<128>(a, x, y, wqkv, wo, wr, grid, s);
    if (dim == 256) return launch_attn<256>(a, x, y, wqkv, wo, wr, grid, s);
    return cudaErrorInvalidValue;
}

}  // namespace prism
