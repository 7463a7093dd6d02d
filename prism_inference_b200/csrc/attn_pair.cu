// attn_pair.cu - the fused window-attention block with every tile split over a cluster of two
// CTAs: the latency path for forwards of few tiles (one 68x120 frame).
//
// Same computation as attn_tc.cu at D = 256 (split2_qkv_attn_d256.comp.glsl:24-79, the router
// of moe_router.comp.glsl:24-52 with N-wide logits), same results bit for bit:
//     y = x + Wo . MHA_window(x) + bo,  assign[t] = argmax_e (Wr . y + br)[e],  counts[e] += 1
// The persistent kernel gives each SM whole 128-row tiles (two 8x8 windows); a frame has only
// 68 of them, so at batch 1 most SMs idle and the serial chain of a tile's eight heads sets the
// time.  Here a cluster of two CTAs takes one tile.  CTA rank r
//   - computes heads 4r..4r+3 (head pairs 2r, 2r+1) for all 128 rows: QKV_h, S_h, softmax,
//     PV_h as attn_tc (the per-row steps of attn_parts.cuh);
//   - owns window r: the out-projection, residual, y store and router of rows [64r, 64r + 64).
// The attention output O of a head pair is therefore needed by both CTAs: the threads of the
// peer's window rows write their O_h rows straight into the peer's shared memory with st.async
// as each head finishes (a landing buffer per head pair, 64 rows x 128 B), and the stores
// complete as transaction bytes on the peer's mbarrier of that pair; the peer's MMAs read the
// rows in place.  No staging, no end-of-loop copy, no y exchange.
// The out-projection accumulates the head pairs in the order 0, 1, 2, 3 on both CTAs, as
// attn_tc does, so the fp32 sums round alike: rank 0 adds its own pairs 0, 1 while its heads
// run and the peer's 2, 3 as they land; rank 1 adds the peer's pair 0 while its heads run, then
// pair 1 when it lands and its own pairs 2, 3, whose window rows it kept.  An M = 128 MMA whose
// A rows of the other window are not needed reads them from whatever lies before or after the
// needed 8 KB (those PO rows are never used).
// All waits are bounded (common.cuh); on timeout a CTA sets the error word and winds down, and
// its peer's waits for it time out likewise.  No TMA multicast.
//
// Warp roles (320 threads) as attn_tc: producer, MMA issuer, softmax group (warps 2-5) and drain
// group (warps 6-9); the y epilogue and the router argmax run on the warps whose TMEM lanes are
// the rows of the CTA's window.  The QKV biases are read through L1; the out-projection and
// router biases are staged in shared memory (the router's as fp16, the blob's own precision).
#include "attn_parts.cuh"
#include "attn_tc.cuh"
#include "common.cuh"

namespace prism {
namespace {

constexpr int kThreads = 320;
constexpr int kStages = 2;
constexpr int kHeads = 4;             // heads per CTA (8 heads of 32 over the pair)
constexpr int kRouterRows = 96;       // router rows per ring stage
constexpr int kStage = 96 * 128 * 4;  // a head's Wqkv rows at full K (48 KB); Wo: 256 rows x 128 B
// shared-memory map (offsets from the 1024-aligned base)
constexpr int kOffX = 0;               // 4 K-blocks x [128][128 B] SW128; y overwrites its own rows
constexpr int kOffQ = kOffX + 65536;   // Q_h [128][64 B] SW64
constexpr int kOffK = kOffQ + 8192;    // K_h
constexpr int kOffV = kOffK + 8192;    // V_h, 2 buffers (head parity)
constexpr int kOffAO = kOffV + 16384;  // rank 0: the current pair's O (SW128 K-block); rank 1: its
                                       //   own window rows of both pairs (8 KB each)
constexpr int kOffL = kOffAO + 16384;  // landings: the peer's O rows of this window, pair 0 | pair 1
constexpr int kOffW = kOffL + 16384;   // weight ring
constexpr int kOffBar = kOffW + kStages * kStage;

// TMEM columns (as attn_tc)
constexpr uint32_t kTPO = 0;     // out-projection accumulator [256]; router logits reuse [0, npad)
constexpr uint32_t kTQKV = 256;  // QKV_h [96]
constexpr uint32_t kTS = 352;    // S_h [128]; P_h over [352, 416)
constexpr uint32_t kTO = 480;    // PV_h [32]

struct Bars {
    uint64_t full[kStages], empty[kStages];
    uint64_t x_full[4], qkv_full, qkv_drained, s_full, p_ready, o_full, o_drained, ao_ready, ao_free;
    // land[p]: the peer's 64 O rows of head pair p landed here (8 KB of st.async transactions);
    // ao_staged: (rank 1) its own window rows of both pairs are written
    uint64_t land[2], ao_staged, po_full, y_ready[4], lg_full, drain, ep_done;
    uint32_t tmem_base;
    int abort;
    float bo[256];
    __half br[256];
    int hist[256];
};
// No alignment slack: the dynamic shared memory of a kernel without static shared memory starts
// 1024-aligned (checked at run time; a misaligned base would end the launch with an error).
constexpr int kSmem = kOffBar + (int)sizeof(Bars);
static_assert(kSmem <= 232448, "shared memory budget");

struct Counter {
    uint32_t n = 0;
    PRISM_DEV uint32_t next() { return (n++) & 1u; }
};

__global__ void __launch_bounds__(kThreads, 1)
    attn_pair_kernel(const AttnTcArgs a, const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_y, const __grid_constant__ CUtensorMap tm_wqkv,
                     const __grid_constant__ CUtensorMap tm_wo, const __grid_constant__ CUtensorMap tm_wr) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw;
    if (smem_u32(smem) & 1023u) {  // the same in both CTAs of the cluster: both leave here
        if (threadIdx.x == 0) atomicOr(a.err, ERR_TIMEOUT);
        return;
    }
    unsigned char* sX = smem + kOffX;
    unsigned char* sQ = smem + kOffQ;
    unsigned char* sK = smem + kOffK;
    unsigned char* sV = smem + kOffV;
    unsigned char* sAO = smem + kOffAO;
    unsigned char* sW = smem + kOffW;
    Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
    volatile int* abort = &bars->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank(), peer = rank ^ 1u;
    const int tile = blockIdx.x >> 1;  // clusters of two consecutive CTAs
    const int wx_n = (a.W + 7) >> 3, wy_n = (a.H + 7) >> 3;
    const int win_per_frame = wx_n * wy_n;
    const int n_windows = win_per_frame * a.frames;
    const int my_w = 2 * tile + (int)rank;  // this CTA's window
    const bool router = a.n_experts > 0;
    const int npad = a.n_experts_pad;
    // The SW128 K-block (128 rows) whose rows of window w are the 8 KB at `rows8k`
    auto kblock_of = [](uint32_t rows8k, uint32_t w) { return rows8k - 8192u * w; };
    const uint32_t landing = smem_u32(smem + kOffL);  // pair p at + 8 KB * p

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int kb = 0; kb < 4; ++kb) {
            mbar_init(&bars->x_full[kb], 1);
            mbar_init(&bars->y_ready[kb], 4);  // the 4 warps on this CTA's window rows
        }
        mbar_init(&bars->qkv_full, 1);
        mbar_init(&bars->qkv_drained, 4);
        mbar_init(&bars->s_full, 1);
        mbar_init(&bars->p_ready, 4);
        mbar_init(&bars->o_full, 1);
        mbar_init(&bars->o_drained, 4);
        mbar_init(&bars->ao_ready, 4);
        mbar_init(&bars->ao_free, 1);
        mbar_init(&bars->ao_staged, 4);
        mbar_init(&bars->po_full, 1);
        mbar_init(&bars->lg_full, 1);
        mbar_init(&bars->drain, 1);
        mbar_init(&bars->ep_done, 4);
        for (int p = 0; p < 2; ++p) {
            mbar_init(&bars->land[p], 1);
            mbar_expect_tx(&bars->land[p], 8192);  // the peer's st.async bytes complete the phase
        }
        bars->abort = 0;
        fence_barrier_init();
        fence_async_shared();
    }
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        bars->hist[i] = 0;
        bars->bo[i] = a.bo[i];
        bars->br[i] = __float2half_rn(router && i < a.n_experts ? a.br[i] : 0.0f);  // exact: fp16 values
    }
    if (warp == 1) tmem_alloc(&bars->tmem_base, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    cluster_sync();  // both CTAs' barriers are initialised before either stores into the other
    const uint32_t tmem = bars->tmem_base;
    // Programmatic dependent launch as attn_tc: the next kernel may place its CTAs now; the wait
    // for the previous kernels is taken by the producer after its first weight loads and by the
    // drain group (routing outputs).
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
            bool ok = true;
            auto ring_load = [&](const CUtensorMap* map, bool kb3d, int c0, int c1, uint32_t bytes) {
                if (!ok || !mbar_wait(&bars->empty[stage], phase ^ 1, abort)) {
                    ok = false;
                    return;
                }
                mbar_expect_tx(&bars->full[stage], bytes);
                if (kb3d)
                    tma_load_3d(smem_u32(sW + stage * kStage), map, &bars->full[stage], 0, c1, 0);
                else
                    tma_load_2d(smem_u32(sW + stage * kStage), map, &bars->full[stage], c0, c1);
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1;
                }
            };
            auto wait = [&](uint64_t* bar, uint32_t par) {
                if (ok && !mbar_wait(bar, par, abort)) ok = false;
            };
            int wf[2], wxx[2], wyy[2];
            for (int half = 0; half < 2; ++half) {
                const int w = 2 * tile + half;
                // a missing second window loads an out-of-range frame: zero fill
                wf[half] = w < n_windows ? w / win_per_frame : a.frames;
                const int wl = w < n_windows ? w % win_per_frame : 0;
                wyy[half] = wl / wx_n;
                wxx[half] = wl % wx_n;
            }
            constexpr uint32_t kQkvBytes = 96 * 128 * 4, kWoBytes = 256 * 128;
            ring_load(&tm_wqkv, true, 0, kHeads * rank * 96, kQkvBytes);
            ring_load(&tm_wqkv, true, 0, (kHeads * rank + 1) * 96, kQkvBytes);
            grid_dep_wait();  // x comes from the previous kernel; y overwrites its input
            for (int kb = 0; kb < 4; ++kb) {
                mbar_expect_tx(&bars->x_full[kb], 16384);
                for (int half = 0; half < 2; ++half)
                    tma_load_4d(smem_u32(sX + kb * 16384 + half * 8192), &tm_x, &bars->x_full[kb], kb * 64,
                                wxx[half] * 8, wyy[half] * 8, wf[half]);
            }
            // the consumption order of the MMA warp: QKV_{h+1} at head h, Wo columns of pair 0 at
            // head 2 (rank 0: its own; rank 1: the peer's), then pairs 1, 2, 3 at the end
            ring_load(&tm_wqkv, true, 0, (kHeads * rank + 2) * 96, kQkvBytes);
            ring_load(&tm_wqkv, true, 0, (kHeads * rank + 3) * 96, kQkvBytes);
            for (int p = 0; p < 4; ++p) ring_load(&tm_wo, false, p * 64, 0, kWoBytes);
            if (router)
                for (int r0 = 0; r0 < npad; r0 += kRouterRows) {
                    const int rows = npad < kRouterRows ? npad : kRouterRows;
                    ring_load(&tm_wr, true, 0, r0, (uint32_t)rows * 512);
                }
            // y of this CTA's window, K-block by K-block as it is written
            for (int kb = 0; kb < 4 && ok; ++kb) {
                wait(&bars->y_ready[kb], 0);
                if (ok && my_w < n_windows) {
                    const int f = my_w / win_per_frame, wl = my_w % win_per_frame;
                    tma_store_4d(&tm_y, smem_u32(sX + kb * 16384 + rank * 8192), kb * 64, (wl % wx_n) * 8,
                                 (wl / wx_n) * 8, f);
                    tma_store_commit();
                }
            }
            tma_store_wait0();
        }
    } else if (warp == 1) {
        // ============================ MMA issuer ==============================
        const uint32_t id_qkv = idesc_f16(128, 96), id_s = idesc_f16(128, 128),
                       id_pv = idesc_f16(128, 32) | (1u << 16) /* B = V MN-major */, id_po = idesc_f16(128, 256);
        int stage = 0;
        uint32_t phase = 0;
        Counter c_qkvd, c_pr, c_od, c_aor;
        bool ok = true;
        auto ring_wait = [&]() -> uint32_t {
            if (ok && !mbar_wait_w(&bars->full[stage], phase, abort)) ok = false;
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
        // the peer's O rows of pair p have landed (st.async, generic proxy): make them visible to
        // the tensor core's reads
        auto wait_landed = [&](int p) {
            if (ok && !__all_sync(0xffffffffu, mbar_wait_cl(&bars->land[p], 0, abort))) ok = false;
            fence_async_shared();
            tc_fence_after();
        };
        const uint32_t xs = smem_u32(sX);
        auto issue_qkv = [&](bool first) {  // the first: X K-blocks as they land
            const uint32_t b = ring_wait();
            if (ok) {
#pragma unroll 1
                for (int kc = 0; kc < 4; ++kc) {
                    if (first) wait(&bars->x_full[kc], 0);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        mma_f16_ss_w(tmem + kTQKV, sdesc(xs + kc * 16384 + k * 32, SW128),
                                     sdesc(b + kc * 12288 + k * 32, SW128), id_qkv, (kc | k) != 0);
                }
                ring_release();
            }
            mma_commit_w(&bars->qkv_full);
        };
        // PO += O_pair . Wo[:, pair]^T with A = the pair's O (an SW128 K-block at `a_base`), the
        // pairs in the order 0, 1, 2, 3
        bool po_first = true;
        auto po_mmas = [&](uint32_t a_base) {
            const uint32_t b = ring_wait();  // Wo[:, pair]: all 256 output rows
            if (!ok) return;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                mma_f16_ss_w(tmem + kTPO, sdesc(a_base + k * 32, SW128), sdesc(b + k * 32, SW128), id_po,
                             !(po_first && k == 0));
            po_first = false;
            ring_release();
        };
        const uint32_t land_kb0 = kblock_of(landing, rank), land_kb1 = kblock_of(landing + 8192, rank);
        issue_qkv(true);
        for (int h = 0; h < kHeads && ok; ++h) {
            const uint32_t vs = smem_u32(sV + (h & 1) * 8192);
            wait(&bars->qkv_drained, c_qkvd.next());
            // ---- S_h = Q K^T
            for (int k = 0; k < 2; ++k)
                mma_f16_ss_w(tmem + kTS, sdesc(smem_u32(sQ) + k * 32, SW64), sdesc(smem_u32(sK) + k * 32, SW64), id_s,
                             k != 0);
            mma_commit_w(&bars->s_full);
            if (h < kHeads - 1) issue_qkv(false);
            if (h == 2) {  // pair 0, behind QKV_3: rank 0 its own, rank 1 the peer's
                if (rank == 0) {
                    wait(&bars->ao_ready, c_aor.next());
                    po_mmas(smem_u32(sAO));
                    mma_commit_w(&bars->ao_free);
                } else {
                    wait_landed(0);
                    po_mmas(land_kb0);
                }
            }
            wait(&bars->p_ready, c_pr.next());
            if (h > 0) wait(&bars->o_drained, c_od.next());  // O columns free
            // ---- O_h = P V, P (fp16) read from TMEM: 16 keys = 8 columns per MMA
            for (int k = 0; k < 8; ++k)
                mma_f16_ts_w(tmem + kTO, tmem + kTS + k * 8, sdesc(vs + k * 1024, SW64), id_pv, k != 0);
            mma_commit_w(&bars->o_full);
        }
        // ---- pairs 1, 2, 3
        if (rank == 0) {
            wait(&bars->ao_ready, c_aor.next());
            po_mmas(smem_u32(sAO));  // own pair 1
            wait_landed(0);
            po_mmas(land_kb0);       // the peer's pair 2
            wait_landed(1);
            po_mmas(land_kb1);       // the peer's pair 3
        } else {
            wait_landed(1);
            po_mmas(land_kb1);       // the peer's pair 1
            wait(&bars->ao_staged, 0);
            for (int q = 0; q < 2 && ok; ++q) po_mmas(kblock_of(smem_u32(sAO) + q * 8192, 1));  // own 2, 3
        }
        mma_commit_w(&bars->po_full);
        // ---- router logits = y . Wr^T (this window's rows of y are whole here)
        if (router && ok) {
            // logits land in PO columns [0, npad): every y K-block has been read out of TMEM
            for (int kb = 0; kb < 4; ++kb) wait(&bars->y_ready[kb], 0);
            const int r_rows = npad < kRouterRows ? npad : kRouterRows;
            for (int r0 = 0; r0 < npad && ok; r0 += kRouterRows) {
                const uint32_t b = ring_wait();
                if (!ok) break;
                const int n = npad - r0 < r_rows ? npad - r0 : r_rows;
                const uint32_t id_r = idesc_f16(128, n);
#pragma unroll 1
                for (int kc = 0; kc < 4; ++kc) {
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        mma_f16_ss_w(tmem + kTPO + r0, sdesc(xs + kc * 16384 + k * 32, SW128),
                                     sdesc(b + kc * r_rows * 128 + k * 32, SW128), id_r, (kc | k) != 0);
                }
                ring_release();
            }
        }
        mma_commit_w(&bars->lg_full);
        mma_commit_w(&bars->drain);
        mbar_wait_w(&bars->drain, 0, abort);
    } else if (warp < 6) {
        // ============================ softmax group ===========================
        const int quad = warp & 3;
        const int r = quad * 32 + lane;  // tile row = TMEM lane
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const int wnd = r >> 6;  // which window of the tile
        const bool mine = wnd == (int)rank;
        const float c2 = a.scale * 1.4426950408889634f;  // scale * log2(e)
        const int nkeys = a.n_keys;
        Counter c_s, c_o;
        bool ok = true;
        auto wait = [&](uint64_t* bar, uint32_t par) {
            if (ok && !mbar_wait(bar, par, abort)) ok = false;
            tc_fence_after();
        };
        auto arrive = [&](uint64_t* bar) {
            __syncwarp();
            if (lane == 0) mbar_arrive(bar);
        };
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
            // ---- O_h = PV / sum -> fp16: the peer's window rows straight into the peer's landing
            // of the pair; this window's rows to the AO buffer (rank 0: the pair's K-block, read
            // by its out-projection; rank 1: its rows of the pair, kept for the end)
            wait(&bars->o_full, c_o.next());
            if (rank == 0 && mine && h == 2) wait(&bars->ao_free, 0);  // pair 0's out-projection done
            if (!ok) break;
            {
                uint32_t v[32];
                tmem_ld32(tmem + lane_addr + kTO, v);
                tmem_ld_wait();
                uint32_t po[16];
                attn_scale_o(v, inv, po);
                const int p = h >> 1;
                if (mine) {
                    const uint32_t base = rank == 0 ? smem_u32(sAO) : kblock_of(smem_u32(sAO) + p * 8192u, 1);
                    unsigned char* dst = smem + (base - smem_u32(smem));
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        *reinterpret_cast<uint4*>(dst + sw128_off(r, (h & 1) * 4 + c)) =
                            make_uint4(po[4 * c], po[4 * c + 1], po[4 * c + 2], po[4 * c + 3]);
                } else {
                    const uint32_t base = peer_addr(kblock_of(landing + p * 8192u, wnd), peer);
                    const uint32_t bar = peer_addr(smem_u32(&bars->land[p]), peer);
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        st_async_peer(base + sw128_off(r, (h & 1) * 4 + c), po[4 * c], po[4 * c + 1], po[4 * c + 2],
                                      po[4 * c + 3], bar);
                }
            }
            fence_async_shared();
            tc_fence_before();
            arrive(&bars->o_drained);
            if ((h & 1) && rank == 0) arrive(&bars->ao_ready);
        }
        arrive(&bars->ao_staged);
        // ---- y: the odd 32-column chunk of every K-block, this CTA's window rows
        if (mine) {
            wait(&bars->po_full, 0);
            if (ok) y_share<4>(sX, tmem + lane_addr + kTPO, r, bars->bo, 1, bars->y_ready, lane);
        }
    } else {
        // ============================ drain group =============================
        const int quad = warp & 3;
        const int r = quad * 32 + lane;  // tile row = TMEM lane
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const int wnd = r >> 6;
        const bool mine = wnd == (int)rank;
        const int li = r & 63;
        const int ty = li >> 3, tx = li & 7;
        Counter c_qkv;
        bool ok = true;
        auto wait = [&](uint64_t* bar, uint32_t par) {
            if (ok && !mbar_wait(bar, par, abort)) ok = false;
            tc_fence_after();
        };
        auto arrive = [&](uint64_t* bar) {
            __syncwarp();
            if (lane == 0) mbar_arrive(bar);
        };
        grid_dep_wait();  // the routing outputs of the previous block are consumed
        for (int h = 0; h < kHeads && ok; ++h) {
            // QKV_h (TMEM) -> fp16 Q, K (K-major SW64) and V (key-major SW64, buffer h&1)
            wait(&bars->qkv_full, c_qkv.next());
            if (!ok) break;
            attn_drain_row(tmem + lane_addr + kTQKV, a.bqkv + (kHeads * rank + h) * 96, r, sQ, sK, sV + (h & 1) * 8192);
            fence_async_shared();
            tc_fence_before();
            arrive(&bars->qkv_drained);
        }
        if (mine) {
            // ---- y: the even 32-column chunk of every K-block, this CTA's window rows
            wait(&bars->po_full, 0);
            if (ok) y_share<4>(sX, tmem + lane_addr + kTPO, r, bars->bo, 0, bars->y_ready, lane);
            // ---- router: logits (PO columns [0, npad)) = fp16(y . Wr^T + br), first maximum
            if (router) {
                wait(&bars->lg_full, 0);
                if (ok && my_w < n_windows) {
                    const int f = my_w / win_per_frame, wl = my_w % win_per_frame;
                    const int gy = (wl / wx_n) * 8 + ty, gx = (wl % wx_n) * 8 + tx;
                    const __half* br = bars->br;
                    const int best = router_argmax(tmem + lane_addr + kTPO, npad, a.n_experts,
                                                   [br](int e) { return __half2float(br[e]); });
                    route_token(a, bars->hist, gy < a.H && gx < a.W,
                                (int64_t)f * a.W * a.H + (int64_t)gy * a.W + gx, best, lane);
                }
            }
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
        const uint64_t t0 = globaltimer();  // stores in flight land
        while (globaltimer() - t0 < 1000000ull) {
        }
    }
    __syncwarp();
    cluster_sync();  // neither CTA leaves while the other may still store into it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace

int attn_pair_smem_bytes() { return kSmem; }

cudaError_t launch_attn_pair(const AttnTcArgs& a, const CUtensorMap& x, const CUtensorMap& y, const CUtensorMap& wqkv,
                             const CUtensorMap& wo, const CUtensorMap& wr, int n_tiles, cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(attn_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    return launch_pdl_cluster(attn_pair_kernel, dim3(2 * n_tiles), dim3(kThreads), kSmem, 2, s, a, x, y, wqkv, wo, wr);
}

}  // namespace prism
