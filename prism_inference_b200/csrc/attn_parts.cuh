// attn_parts.cuh - per-row SIMT steps shared by the two tcgen05 window-attention kernels
// (attn_tc.cu: one CTA per 128-row tile; attn_pair.cu: a tile's heads split over a CTA pair).
// Thread = tile row = TMEM lane; every function works on the calling thread's row.
#pragma once
#include "attn_tc.cuh"
#include "common.cuh"

namespace prism {

// Softmax of one row of S over its window's keys (split2_qkv_attn_d256.comp.glsl:59-66):
// s_j = acc_j * scale, p_j = exp(s_j - max s) as 2^(acc_j * scale log2 e - max * scale log2 e)
// (scale > 0, so the maximum of the scaled scores is the scaled maximum).  sv = the row's 64
// scores of its own window; pk = the weights as packed fp16 pairs; returns the fp32 sum.
// Frames of fewer than 64 tokens have n_keys < 64 keys per window (:33).
PRISM_DEV float attn_softmax_row(const uint32_t (&sv)[64], float c2, int nkeys, uint32_t (&pk)[32]) {
    float se;
    if (nkeys >= 64) {
        float m0 = __uint_as_float(sv[0]), m1 = __uint_as_float(sv[1]), m2 = __uint_as_float(sv[2]),
              m3 = __uint_as_float(sv[3]);
#pragma unroll
        for (int j = 4; j < 64; j += 4) {
            m0 = fmaxf(m0, __uint_as_float(sv[j]));
            m1 = fmaxf(m1, __uint_as_float(sv[j + 1]));
            m2 = fmaxf(m2, __uint_as_float(sv[j + 2]));
            m3 = fmaxf(m3, __uint_as_float(sv[j + 3]));
        }
        const float mc = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3)) * c2;
        // the per-key fma(s, scale log2 e, -max) and the four running sums as f32x2 pairs
        // (the same operations per element)
        const uint64_t c22 = f2_pack(c2, c2), nmc = f2_pack(-mc, -mc);
        uint64_t s01 = f2_pack(0.f, 0.f), s23 = f2_pack(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 64; j += 4) {
            float a0, a1, a2, a3;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[j]), __uint_as_float(sv[j + 1])), c22, nmc), a0, a1);
            f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[j + 2]), __uint_as_float(sv[j + 3])), c22, nmc), a2, a3);
            const float p0 = ex2_approx(a0), p1 = ex2_approx(a1), p2 = ex2_approx(a2), p3 = ex2_approx(a3);
            s01 = f2_add(s01, f2_pack(p0, p1));
            s23 = f2_add(s23, f2_pack(p2, p3));
            pk[j >> 1] = pack_h2(p0, p1);
            pk[(j >> 1) + 1] = pack_h2(p2, p3);
        }
        float s0, s1, s2, s3;
        f2_unpack(s01, s0, s1);
        f2_unpack(s23, s2, s3);
        se = (s0 + s1) + (s2 + s3);
    } else {
        // keys are the first n_keys slots of the window
        float m = -1e9f;
#pragma unroll
        for (int j = 0; j < 64; ++j)
            if (j < nkeys) m = fmaxf(m, __uint_as_float(sv[j]));
        const float mc = m * c2;
        se = 0.f;
#pragma unroll
        for (int j = 0; j < 64; j += 2) {
            const float p0 = j < nkeys ? ex2_approx(fmaf(__uint_as_float(sv[j]), c2, -mc)) : 0.f;
            const float p1 = j + 1 < nkeys ? ex2_approx(fmaf(__uint_as_float(sv[j + 1]), c2, -mc)) : 0.f;
            se += p0 + p1;
            pk[j >> 1] = pack_h2(p0, p1);
        }
    }
    return se;
}

// P row into TMEM over S: keys of window A in columns [0, 32), window B in [32, 64); this row's
// keys get the weights, the other window's keys zero (the PV MMA is block-diagonal).
PRISM_DEV void attn_store_p(uint32_t s_taddr, int wnd, const uint32_t (&pk)[32]) {
    uint32_t zero[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) zero[j] = 0u;
    tmem_st32(s_taddr + wnd * 32, pk);
    tmem_st32(s_taddr + (wnd ^ 1) * 32, zero);
    tmem_st_wait();
}

// O row / sum -> 32 fp16 values as 16 packed pairs (f32x2 multiplies)
PRISM_DEV void attn_scale_o(const uint32_t (&v)[32], float inv, uint32_t (&po)[16]) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        float o0, o1;
        f2_unpack(f2_mul(f2_pack(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1])), f2_pack(inv, inv)), o0,
                  o1);
        po[j] = pack_h2(o0, o1);
    }
}

// QKV_h of one row (TMEM, 96 fp32 columns at qkv_taddr) + bias bq[96] -> fp16 Q, K and V rows in
// shared memory, each 32 fp16 = four 16-byte chunks in SW64 layout (V is the MN-major B operand
// of PV, which has exactly this layout, so it is stored like K).
PRISM_DEV void attn_drain_row(uint32_t qkv_taddr, const float* bq, int r, unsigned char* sQ, unsigned char* sK,
                              unsigned char* sV) {
#pragma unroll
    for (int part = 0; part < 3; ++part) {  // Q, K, V
        uint32_t v[32];
        tmem_ld32(qkv_taddr + part * 32, v);
        float4 bb[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) bb[i] = *reinterpret_cast<const float4*>(bq + part * 32 + 4 * i);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            pk[2 * i] = add_pack_h2(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]), bb[i].x, bb[i].y);
            pk[2 * i + 1] = add_pack_h2(__uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]), bb[i].z, bb[i].w);
        }
        unsigned char* dst = part == 0 ? sQ : part == 1 ? sK : sV;
#pragma unroll
        for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(dst + sw64_off(r, c)) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
    }
}

// y = fp16(fp16(PO + bo) + x) for the 32 columns [32g, 32g + 32) of tile row r (v = PO of
// those columns), written over x in its swizzled slot of the K-blocks at sX (bo staged in
// shared memory, indexed like g).
PRISM_DEV void y_chunk(unsigned char* sX, const uint32_t (&v)[32], int r, const float* bo, int g) {
    unsigned char* xblk = sX + (g >> 1) * 16384;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const int off = sw128_off(r, (g & 1) * 4 + c);
        const uint4 x = *reinterpret_cast<const uint4*>(xblk + off);
        const float4 b0 = *reinterpret_cast<const float4*>(bo + g * 32 + 8 * c);
        const float4 b1 = *reinterpret_cast<const float4*>(bo + g * 32 + 8 * c + 4);
        const float* fv = reinterpret_cast<const float*>(&v[8 * c]);
        // y = h( h(PO + bo) + x ): the second rounding is the fp16 add (split2_qkv_attn_d256.comp.glsl:76)
        uint4 y;
        y.x = hadd2_u32(add_pack_h2(fv[0], fv[1], b0.x, b0.y), x.x);
        y.y = hadd2_u32(add_pack_h2(fv[2], fv[3], b0.z, b0.w), x.y);
        y.z = hadd2_u32(add_pack_h2(fv[4], fv[5], b1.x, b1.y), x.z);
        y.w = hadd2_u32(add_pack_h2(fv[6], fv[7], b1.z, b1.w), x.w);
        *reinterpret_cast<uint4*>(xblk + off) = y;
    }
}

// One SIMT group's share of y: chunk 2kb + part of every K-block kb < KB, in order, each K-block
// announced on y_ready[kb] (with the other group's chunk it completes the K-block).  PO is at
// TMEM column 0 of the row (po_taddr).  The TMEM load of the next chunk is in flight while the
// current one is computed; the router GEMM writes logits only over K-blocks already announced,
// so the load in flight is never overwritten.
template <int KB>
PRISM_DEV void y_share(unsigned char* sX, uint32_t po_taddr, int r, const float* bo, int part, uint64_t* y_ready,
                       int lane) {
    uint32_t va[32], vb[32];
    tmem_ld32(po_taddr + part * 32, va);
    tmem_ld_wait();
#pragma unroll
    for (int kb = 0; kb < KB; ++kb) {
        uint32_t(&cur)[32] = (kb & 1) ? vb : va;
        uint32_t(&nxt)[32] = (kb & 1) ? va : vb;
        if (kb < KB - 1) tmem_ld32(po_taddr + (2 * (kb + 1) + part) * 32, nxt);
        y_chunk(sX, cur, r, bo, 2 * kb + part);
        fence_async_shared();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&y_ready[kb]);
        if (kb < KB - 1) tmem_ld_wait();
    }
}

// The router's choice for one row: the first maximum of the logits l_e = fp16(acc_e + br_e),
// e < n_experts (the lowest index among equal maxima, which the sequential scan
// `if (e == 0 || l > best)` of moe_router.comp.glsl picks), with acc_e in TMEM columns [0, npad)
// at taddr and br_e = bias(e).  The 32 logits of a TMEM load are rounded independently and
// reduced as a tree in which the higher index of a pair wins only when strictly greater (so ties
// keep the lower index); batches of 32 combine the same way.  A serial scan would be a chain of
// 64 dependent compare-selects at 64 experts.
template <typename Bias>
PRISM_DEV int router_argmax(uint32_t taddr, int npad, int n_experts, Bias bias) {
    float bv = 0.0f;
    int best = 0;
#pragma unroll 1
    for (int g = 0; g < npad; g += 32) {
        uint32_t v[32];
        if (g + 32 <= npad) {
            tmem_ld32(taddr + g, v);
        } else {  // npad is a multiple of 16: the last 16 columns
            tmem_ld16(taddr + g, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
#pragma unroll
            for (int j = 16; j < 32; ++j) v[j] = 0u;
        }
        tmem_ld_wait();
        float l[32];
        int id[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            l[j] = g + j < n_experts ? rh(__fadd_rn(__uint_as_float(v[j]), bias(g + j))) : -INFINITY;
            id[j] = g + j;
        }
#pragma unroll
        for (int s = 1; s < 32; s <<= 1)
#pragma unroll
            for (int j = 0; j < 32; j += 2 * s)
                if (l[j + s] > l[j]) {
                    l[j] = l[j + s];
                    id[j] = id[j + s];
                }
        if (g == 0 || l[0] > bv) {
            bv = l[0];
            best = id[0];
        }
    }
    return best;
}

// Record the expert e of a routed token (valid: this lane's row is a token of the frame):
// assign[token] = e, then either the CTA histogram (added to counts once per CTA; the route
// kernel builds the permutation from counts) or the token's slot in expert e's bucket, with
// counts[e] as the bucket cursor: one atomic per expert and warp, lanes ranked by lane index.
// Called by the active lanes of the warp together.  A slot past the bucket capacity (counts left behind by a
// forward that gave up) is not written and raises ERR_ROUTE.
PRISM_DEV void route_token(const AttnTcArgs& a, int* hist, bool valid, int64_t token, int e, int lane) {
    const uint32_t vm = __ballot_sync(__activemask(), valid);
    if (!valid) return;
    a.assign[token] = e;
    if (!a.perm_b) {
        atomicAdd(&hist[e], 1);
        return;
    }
    const uint32_t peers = __match_any_sync(vm, e);
    const int leader = __ffs(peers) - 1;
    int base = 0;
    if (lane == leader) base = atomicAdd(&a.counts[e], __popc(peers));
    base = __shfl_sync(peers, base, leader);
    const int k = base + __popc(peers & ((1u << lane) - 1u));
    if (k < a.perm_stride)
        a.perm_b[(int64_t)e * a.perm_stride + k] = (int32_t)token;
    else
        atomicOr(a.err, ERR_ROUTE);
}

}  // namespace prism
