// pkv_attn.cu -- fused dequantize + flash-decoding attention over packed codes.
//
// Computes, per batch row b and query head h (one query token),
//     out = softmax(q' . Khat^T * scale) . Vhat @ R,      q' = q @ R^T,
// where Khat/Vhat are the rotated-space triplets decoded from the packed
// K/V codes.  This equals PolarAttentionApprox.forward with decoded values
// (polar_attention.py:277-309; the polar identity of :113-212 is the dot
// product with the decoded key) and the decode-then-attend composite for
// learned codebooks / BiasTable / Lloyd-Max (stacked_plane.py:268-327),
// because decode = rot_q @ R and R is orthogonal.
//
// Layout and schedule:
//  * codes: (B, Hkv, S, m) of uint8/uint16, one 32/64-byte row per token;
//  * one work item = (b, kv head, split) = a contiguous token range;
//    persistent CTAs take items round-robin;
//  * warp 4 (producer) streams K and V code tiles of TT tokens into a
//    STAGES-deep shared-memory ring with 1-D TMA bulk copies completing on
//    mbarriers; warps 0-3 (consumers) each own 32 tokens of a tile;
//  * consumer lane j owns triplet j (and j+32): it decodes the code through
//    the shared-memory LUT and forms partial dot products for every query
//    head of the group; a 32-way transpose-reduce leaves the full score of
//    one (head, token) pair in each lane; online softmax in base 2; V is
//    accumulated per lane in rotated space (no reduction needed);
//  * splits of one (b, kv head) write (m, l, o) partials to the workspace;
//    the last CTA to finish (atomic counter) merges them, normalises and
//    applies R once, then resets the counter.
//
// Every mbarrier wait is bounded; on expiry the kernel sets the device error
// word, stops issuing copies, drains what it issued and returns.

#include <algorithm>
#include <cmath>

#include "pkv_common.cuh"

namespace pkv {

constexpr int kConsumerWarps = 4;
constexpr int kTT = 128;               // tokens per tile (32 per consumer warp)
constexpr float kLn2 = 0.69314718055994530942f;

struct AttnParams {
    int B, Hq, Hkv, S, G, m, dim;
    const void* q; int qdt; int64_t q_bs, q_hs;
    const uint8_t* kc; const uint8_t* vc;
    int64_t kv_bs, kv_hs;              // in codes
    const int32_t* seq_lens;
    float scale_log2;
    float* out; int64_t out_bs, out_hs;
    int nsplit, chunk;                 // chunk: tokens per split, multiple of kTT
    int partial_only; float* partial_out;
    float* ws_part; int32_t* ws_count;
    const float* R; const float* dec_z; const float* dec_xy;
    int bits_flat, code_mask, flat_mask, xy_per_z, n_xy, Cz;
    int num_items, stages;
    float* sm_dummy;
};

struct SmemLayout {
    int stage_bytes, stages;
    int off_stage, off_R, off_xy, off_z, off_q, off_cm, off_cl, off_co, off_fin, off_bar, off_flag, total;
};

__host__ __device__ inline int align_up(int x, int a) { return (x + a - 1) / a * a; }

__host__ __device__ inline SmemLayout attn_smem_layout(int m, int cb, int dim, int G, int n_xy, int Cz, int stages) {
    SmemLayout L;
    L.stages = stages;
    L.stage_bytes = 2 * kTT * m * cb;
    int o = 0;
    L.off_stage = o; o += stages * L.stage_bytes; o = align_up(o, 16);
    L.off_R = o; o += dim * (dim + 1) * 4; o = align_up(o, 16);
    L.off_xy = o; o += n_xy * 8; o = align_up(o, 16);
    L.off_z = o; o += Cz * 4; o = align_up(o, 16);
    L.off_q = o; o += G * dim * 4; o = align_up(o, 16);
    L.off_cm = o; o += kConsumerWarps * G * 4;
    L.off_cl = o; o += kConsumerWarps * G * 4; o = align_up(o, 16);
    L.off_co = o; o += kConsumerWarps * G * dim * 4; o = align_up(o, 16);
    L.off_fin = o; o += G * dim * 4; o = align_up(o, 16);
    L.off_bar = o; o += 2 * stages * 8;
    L.off_flag = o; o += 16;
    L.total = o;
    return L;
}

__device__ __forceinline__ float q_load(const void* q, int qdt, int64_t idx) {
    if (qdt == PKV_F32) return __ldg(static_cast<const float*>(q) + idx);
    if (qdt == PKV_BF16) return __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(q) + idx));
    return __half2float(__ldg(static_cast<const __half*>(q) + idx));
}

struct ItemRange { int b, hk, split, tok0, tok1; };

__device__ __forceinline__ ItemRange item_range(const AttnParams& p, int item) {
    ItemRange r;
    r.split = item % p.nsplit;
    int bh = item / p.nsplit;
    r.hk = bh % p.Hkv;
    r.b = bh / p.Hkv;
    int L = p.seq_lens ? min(max(p.seq_lens[r.b], 0), p.S) : p.S;
    r.tok0 = r.split * p.chunk;
    r.tok1 = min(L, r.tok0 + p.chunk);
    if (r.tok1 < r.tok0) r.tok1 = r.tok0;
    return r;
}

// transpose-reduce: on entry each lane holds v[0..31]; on exit v[0] of lane l
// holds sum over all lanes of their v[l].
__device__ __forceinline__ void transpose_reduce32(float (&v)[32], int lane) {
    #pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const bool upper = (lane & off) != 0;
        #pragma unroll
        for (int i = 0; i < off; ++i) {
            float send = upper ? v[i] : v[i + off];
            float keep = upper ? v[i + off] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
}

template <int CB, int TPL, int G, bool TMA>
__global__ void __launch_bounds__(TMA ? 160 : 128) attn_decode_kernel(AttnParams p) {
    using CT = typename Code<CB>::T;
    constexpr int TB = 32 / G;                     // tokens per transpose block
    extern __shared__ __align__(128) uint8_t attn_smem[];
    uint8_t* smem = attn_smem;
    const SmemLayout L = attn_smem_layout(p.m, CB, p.dim, G, p.n_xy, p.Cz, p.stages);
    float* sR = reinterpret_cast<float*>(smem + L.off_R);          // R[k][i], pitch dim+1
    const float2* sXY = reinterpret_cast<const float2*>(smem + L.off_xy);
    const float* sZ = reinterpret_cast<const float*>(smem + L.off_z);
    float* sQ = reinterpret_cast<float*>(smem + L.off_q);          // [G][dim]
    float* sCm = reinterpret_cast<float*>(smem + L.off_cm);        // [4][G]
    float* sCl = reinterpret_cast<float*>(smem + L.off_cl);        // [4][G]
    float* sCo = reinterpret_cast<float*>(smem + L.off_co);        // [4][G][dim]
    float* sFin = reinterpret_cast<float*>(smem + L.off_fin);      // [G][dim]
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.off_bar);
    uint64_t* empty = full + p.stages;
    int* sflag = reinterpret_cast<int*>(smem + L.off_flag);

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int dim = p.dim, m = p.m, pitch = dim + 1;
    const int nthreads = blockDim.x;

    // ---- prologue: R, LUTs, barriers --------------------------------------
    for (int idx = tid; idx < dim * dim; idx += nthreads) {
        int k = idx / dim, i = idx % dim;
        sR[k * pitch + i] = __ldg(p.R + idx);
    }
    {
        float2* xy = reinterpret_cast<float2*>(smem + L.off_xy);
        const float2* g = reinterpret_cast<const float2*>(p.dec_xy);
        for (int idx = tid; idx < p.n_xy; idx += nthreads) xy[idx] = __ldg(g + idx);
        float* z = reinterpret_cast<float*>(smem + L.off_z);
        for (int idx = tid; idx < p.Cz; idx += nthreads) z[idx] = __ldg(p.dec_z + idx);
    }
    if (TMA && tid == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_mbar_init();
    }
    if (tid == 0) sflag[1] = 0;                    // sticky abort flag for this CTA
    __syncthreads();

    // ---- producer warp ------------------------------------------------------
    if (TMA && warp == kConsumerWarps) {
        if (lane == 0) {
            const uint32_t row_bytes = (uint32_t)(m * CB);
            int seq = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < p.num_items && ok; item += gridDim.x) {
                ItemRange r = item_range(p, item);
                const int64_t base = ((int64_t)r.b * p.kv_bs + (int64_t)r.hk * p.kv_hs) * CB;
                for (int t0 = r.tok0; t0 < r.tok1; t0 += kTT, ++seq) {
                    const int s = seq % p.stages;
                    const int use = seq / p.stages;
                    if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, kErrWaitEmpty)) { ok = false; break; }
                    const int nt = min(kTT, r.tok1 - t0);
                    const uint32_t bytes = (uint32_t)nt * row_bytes;
                    uint8_t* dk = smem + L.off_stage + s * L.stage_bytes;
                    uint8_t* dv = dk + kTT * row_bytes;
                    mbar_arrive_expect_tx(&full[s], 2 * bytes);
                    bulk_g2s(dk, p.kc + base + (int64_t)t0 * row_bytes, bytes, &full[s]);
                    bulk_g2s(dv, p.vc + base + (int64_t)t0 * row_bytes, bytes, &full[s]);
                }
            }
            // drain: every issued copy must land before the CTA may exit
            const int issued = seq;
            for (int q = max(0, issued - p.stages); q < issued; ++q)
                mbar_wait(&full[q % p.stages], (q / p.stages) & 1, kErrWaitDrain);
        }
        return;
    }

    // ---- consumers ----------------------------------------------------------
    const int myh = lane / TB, myt = lane % TB;
    int seq = 0;
    bool alive = true;
    for (int item = blockIdx.x; item < p.num_items; item += gridDim.x) {
        const ItemRange r = item_range(p, item);
        const int greal = p.G;
        // rotated, scaled query of every head of the group -> sQ
        for (int idx = tid; idx < G * dim; idx += kConsumerWarps * 32) {
            int g = idx / dim, k = idx % dim;
            float acc = 0.f;
            if (g < greal) {
                const int hq = r.hk * greal + g;
                const int64_t qb = (int64_t)r.b * p.q_bs + (int64_t)hq * p.q_hs;
                #pragma unroll 4
                for (int i = 0; i < dim; ++i) acc = fmaf(q_load(p.q, p.qdt, qb + i), sR[k * pitch + i], acc);
            }
            sQ[idx] = acc * p.scale_log2;
        }
        named_bar_sync(1, kConsumerWarps * 32);
        float qv[G][TPL][3];
        #pragma unroll
        for (int g = 0; g < G; ++g)
            #pragma unroll
            for (int tp = 0; tp < TPL; ++tp) {
                int j = lane + 32 * tp;
                #pragma unroll
                for (int c = 0; c < 3; ++c) qv[g][tp][c] = (j < m) ? sQ[g * dim + 3 * j + c] : 0.f;
            }
        float acc[G][TPL][3];
        float mrun[G];
        #pragma unroll
        for (int g = 0; g < G; ++g) {
            mrun[g] = -INFINITY;
            #pragma unroll
            for (int tp = 0; tp < TPL; ++tp) acc[g][tp][0] = acc[g][tp][1] = acc[g][tp][2] = 0.f;
        }
        float lrun = 0.f;
        const int64_t base = (int64_t)r.b * p.kv_bs + (int64_t)r.hk * p.kv_hs;   // codes

        for (int t0 = r.tok0; t0 < r.tok1; t0 += kTT, ++seq) {
            const int s = seq % p.stages;
            const CT* Kt;
            const CT* Vt;
            if (TMA) {
                if (alive && !mbar_wait(&full[s], (seq / p.stages) & 1, kErrWaitFull)) alive = false;
                Kt = reinterpret_cast<const CT*>(smem + L.off_stage + s * L.stage_bytes);
                Vt = Kt + kTT * m;
            } else {
                Kt = reinterpret_cast<const CT*>(p.kc) + base + (int64_t)t0 * m;
                Vt = reinterpret_cast<const CT*>(p.vc) + base + (int64_t)t0 * m;
            }
            const int nt = min(kTT, r.tok1 - t0);
            if (alive) {
                #pragma unroll 1
                for (int blk = 0; blk < 32 / TB; ++blk) {
                    const int tl0 = warp * 32 + blk * TB;      // first token of block in tile
                    if (tl0 >= nt) break;                      // warp-uniform
                    float ps[32];
                    #pragma unroll
                    for (int t = 0; t < TB; ++t) {
                        float part[G];
                        #pragma unroll
                        for (int g = 0; g < G; ++g) part[g] = 0.f;
                        const bool tv = (tl0 + t) < nt;
                        #pragma unroll
                        for (int tp = 0; tp < TPL; ++tp) {
                            const int j = lane + 32 * tp;
                            if (j < m) {
                                uint32_t code = 0;
                                if (tv) code = TMA ? (uint32_t)Kt[(tl0 + t) * m + j]
                                                   : Code<CB>::load(Kt + (tl0 + t) * m + j);
                                code &= p.code_mask;
                                const float z = sZ[code >> p.bits_flat];
                                const float2 xy = sXY[p.xy_per_z ? code : (code & p.flat_mask)];
                                #pragma unroll
                                for (int g = 0; g < G; ++g)
                                    part[g] = fmaf(qv[g][tp][0], z, fmaf(qv[g][tp][1], xy.x, fmaf(qv[g][tp][2], xy.y, part[g])));
                            }
                        }
                        #pragma unroll
                        for (int g = 0; g < G; ++g) ps[g * TB + t] = part[g];
                    }
                    transpose_reduce32(ps, lane);
                    const bool valid = (tl0 + myt) < nt && myh < greal;
                    float sc = valid ? ps[0] : -INFINITY;
                    float bm = sc;
                    #pragma unroll
                    for (int off = TB / 2; off >= 1; off >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, off));
                    float alpha_mine = 1.f;
                    #pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float mn = fmaxf(mrun[g], __shfl_sync(0xffffffffu, bm, g * TB));
                        if (mn != mrun[g]) {                   // warp-uniform
                            const float alpha = fast_exp2(mrun[g] - mn);   // 0 when mrun = -inf
                            #pragma unroll
                            for (int tp = 0; tp < TPL; ++tp) {
                                acc[g][tp][0] *= alpha; acc[g][tp][1] *= alpha; acc[g][tp][2] *= alpha;
                            }
                            if (g == myh) alpha_mine = alpha;
                            mrun[g] = mn;
                        }
                    }
                    float mine_m = mrun[0];
                    #pragma unroll
                    for (int g = 1; g < G; ++g) if (g == myh) mine_m = mrun[g];
                    const float pr = valid ? fast_exp2(sc - mine_m) : 0.f;
                    lrun = lrun * alpha_mine + pr;
                    // V
                    #pragma unroll
                    for (int t = 0; t < TB; ++t) {
                        float pg[G];
                        #pragma unroll
                        for (int g = 0; g < G; ++g) pg[g] = __shfl_sync(0xffffffffu, pr, g * TB + t);
                        const bool tv = (tl0 + t) < nt;
                        #pragma unroll
                        for (int tp = 0; tp < TPL; ++tp) {
                            const int j = lane + 32 * tp;
                            if (j < m) {
                                uint32_t code = 0;
                                if (tv) code = TMA ? (uint32_t)Vt[(tl0 + t) * m + j]
                                                   : Code<CB>::load(Vt + (tl0 + t) * m + j);
                                code &= p.code_mask;
                                const float z = sZ[code >> p.bits_flat];
                                const float2 xy = sXY[p.xy_per_z ? code : (code & p.flat_mask)];
                                #pragma unroll
                                for (int g = 0; g < G; ++g) {
                                    acc[g][tp][0] = fmaf(pg[g], z, acc[g][tp][0]);
                                    acc[g][tp][1] = fmaf(pg[g], xy.x, acc[g][tp][1]);
                                    acc[g][tp][2] = fmaf(pg[g], xy.y, acc[g][tp][2]);
                                }
                            }
                        }
                    }
                }
            }
            if (TMA) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
        }

        // ---- per-item epilogue: merge the 4 consumer warps ---------------------
        float lsum = lrun;
        #pragma unroll
        for (int off = TB / 2; off >= 1; off >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
        #pragma unroll
        for (int g = 0; g < G; ++g) {
            const float lg = __shfl_sync(0xffffffffu, lsum, g * TB);
            if (lane == 0) { sCm[warp * G + g] = mrun[g]; sCl[warp * G + g] = lg; }
            #pragma unroll
            for (int tp = 0; tp < TPL; ++tp) {
                int j = lane + 32 * tp;
                if (j < m) {
                    float* o = sCo + (warp * G + g) * dim + 3 * j;
                    o[0] = acc[g][tp][0]; o[1] = acc[g][tp][1]; o[2] = acc[g][tp][2];
                }
            }
        }
        named_bar_sync(1, kConsumerWarps * 32);
        const bool single = (p.nsplit == 1);
        // merge warps: (g, k) pairs; write partial row or normalised result
        for (int idx = tid; idx < G * (dim + 2); idx += kConsumerWarps * 32) {
            const int g = idx / (dim + 2), k = idx % (dim + 2);
            if (g >= greal) continue;
            float M = -INFINITY;
            #pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sCm[w * G + g]);
            float v = 0.f, lsw = 0.f;
            #pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
                const float mw = sCm[w * G + g];
                const float f = (mw == -INFINITY) ? 0.f : fast_exp2(mw - M);
                lsw = fmaf(sCl[w * G + g], f, lsw);
                if (k >= 2) v = fmaf(sCo[(w * G + g) * dim + (k - 2)], f, v);
            }
            const int hq = r.hk * greal + g;
            if (single && !p.partial_only) {
                if (k >= 2) sFin[g * dim + (k - 2)] = (lsw > 0.f) ? v / lsw : 0.f;
            } else {
                const float val = (k == 0) ? M : (k == 1 ? lsw : v);
                if (single) {
                    float* dst = p.partial_out + ((int64_t)r.b * p.Hq + hq) * (dim + 2);
                    dst[k] = (k == 0) ? (M == -INFINITY ? -INFINITY : M * kLn2) : val;
                } else {
                    float* dst = p.ws_part + (((int64_t)r.b * p.Hq + hq) * p.nsplit + r.split) * (dim + 2);
                    dst[k] = val;                                     // log2-domain max
                }
            }
        }
        bool finalize = single && !p.partial_only;
        bool merge_splits = false;
        if (!single) {
            __threadfence();
            named_bar_sync(1, kConsumerWarps * 32);
            if (tid == 0) {
                int32_t* cnt = p.ws_count + (r.b * p.Hkv + r.hk);
                const int prev = atomicAdd(cnt, 1);
                const int last = (prev == p.nsplit - 1);
                if (last) { __threadfence(); atomicExch(cnt, 0); }
                sflag[0] = last;
            }
            named_bar_sync(1, kConsumerWarps * 32);
            merge_splits = sflag[0] != 0;
            if (merge_splits) {
                for (int idx = tid; idx < G * (dim + 2); idx += kConsumerWarps * 32) {
                    const int g = idx / (dim + 2), k = idx % (dim + 2);
                    if (g >= greal) continue;
                    const int hq = r.hk * greal + g;
                    const float* src = p.ws_part + ((int64_t)r.b * p.Hq + hq) * p.nsplit * (dim + 2);
                    float M = -INFINITY;
                    for (int sp = 0; sp < p.nsplit; ++sp) M = fmaxf(M, __ldcg(src + sp * (dim + 2)));
                    float v = 0.f, lsw = 0.f;
                    for (int sp = 0; sp < p.nsplit; ++sp) {
                        const float ms = __ldcg(src + sp * (dim + 2));
                        const float f = (ms == -INFINITY) ? 0.f : fast_exp2(ms - M);
                        lsw = fmaf(__ldcg(src + sp * (dim + 2) + 1), f, lsw);
                        if (k >= 2) v = fmaf(__ldcg(src + sp * (dim + 2) + k), f, v);
                    }
                    if (p.partial_only) {
                        float* dst = p.partial_out + ((int64_t)r.b * p.Hq + hq) * (dim + 2);
                        dst[k] = (k == 0) ? (M == -INFINITY ? -INFINITY : M * kLn2) : (k == 1 ? lsw : v);
                    } else if (k >= 2) {
                        sFin[g * dim + (k - 2)] = (lsw > 0.f) ? v / lsw : 0.f;
                    }
                }
                finalize = !p.partial_only;
            }
        }
        if (finalize) {
            named_bar_sync(1, kConsumerWarps * 32);
            // out = fin @ R   (R[k][i], pitch dim+1: lanes over i are conflict-free)
            for (int idx = tid; idx < greal * dim; idx += kConsumerWarps * 32) {
                const int g = idx / dim, i = idx % dim;
                float v = 0.f;
                #pragma unroll 4
                for (int k = 0; k < dim; ++k) v = fmaf(sFin[g * dim + k], sR[k * pitch + i], v);
                const int hq = r.hk * greal + g;
                p.out[(int64_t)r.b * p.out_bs + (int64_t)hq * p.out_hs + i] = v;
            }
        }
        named_bar_sync(1, kConsumerWarps * 32);     // smem scratch reused by the next item
    }
}

// ---------------------------------------------------------------------------
// cross-shard log-sum-exp merge (+ normalise + R)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) lse_combine_kernel(const float* __restrict__ parts, int n_parts,
                                                          int64_t part_stride, int rows, int dim,
                                                          const float* __restrict__ R,
                                                          float* __restrict__ out, int64_t out_rs) {
    extern __shared__ float fin[];                 // [dim]
    const int row = blockIdx.x;
    if (row >= rows) return;
    for (int k = threadIdx.x; k < dim; k += blockDim.x) {
        float M = -INFINITY;
        for (int pi = 0; pi < n_parts; ++pi) M = fmaxf(M, __ldg(parts + pi * part_stride + (int64_t)row * (dim + 2)));
        float l = 0.f, v = 0.f;
        for (int pi = 0; pi < n_parts; ++pi) {
            const float* src = parts + pi * part_stride + (int64_t)row * (dim + 2);
            const float mp = __ldg(src);
            const float f = (mp == -INFINITY) ? 0.f : expf(mp - M);
            l = fmaf(__ldg(src + 1), f, l);
            v = fmaf(__ldg(src + 2 + k), f, v);
        }
        fin[k] = (l > 0.f) ? v / l : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        float v = 0.f;
        for (int k = 0; k < dim; ++k) v = fmaf(fin[k], __ldg(R + k * dim + i), v);
        out[(int64_t)row * out_rs + i] = v;
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static int num_sms() {
    static int cached = 0;
    if (!cached) {
        int dev = 0, n = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = PKV_NUM_SMS_B200;
        cached = n;
    }
    return cached;
}

static int round_group(int G) { return G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8; }

struct AttnPlan {
    int G, TPL, stages, nsplit, chunk;
    bool tma;
    SmemLayout L;
};

static AttnPlan plan_attn(const pkv_codec* c, const pkv_attn_args* a) {
    AttnPlan pl{};
    const int m = c->dim / 3;
    const int g = a->q_heads / a->kv_heads;
    pl.G = round_group(g);
    pl.TPL = (m <= 32) ? 1 : 2;
    const int row_bytes = m * a->code_bytes;
    pl.stages = (row_bytes <= 64) ? 4 : 3;
    const int Cz = 1 << c->bits_z;
    const int n_xy = (c->xy_per_z ? Cz : 1) << (c->bits_r + c->bits_theta);
    pl.L = attn_smem_layout(m, a->code_bytes, c->dim, pl.G, n_xy, Cz, pl.stages);
    while (pl.L.total > 227 * 1024 && pl.stages > 2) {      // large head dims: shallower ring
        --pl.stages;
        pl.L = attn_smem_layout(m, a->code_bytes, c->dim, pl.G, n_xy, Cz, pl.stages);
    }
    // TMA needs 16-byte aligned rows and bases
    const uintptr_t kb = reinterpret_cast<uintptr_t>(a->k_codes), vb = reinterpret_cast<uintptr_t>(a->v_codes);
    pl.tma = (row_bytes % 16 == 0) && (kb % 16 == 0) && (vb % 16 == 0) &&
             ((a->kv_batch_stride * a->code_bytes) % 16 == 0) && ((a->kv_head_stride * a->code_bytes) % 16 == 0);
    // split count: minimise rounds * (tiles per item + overhead)
    const int tiles_total = std::max(1, (a->seq_len + kTT - 1) / kTT);
    const int64_t units = (int64_t)a->batch * a->kv_heads;
    const int64_t grid = (int64_t)num_sms() * 2;
    int best = 1;
    double best_cost = 1e300;
    int max_split = a->num_splits > 0 ? a->num_splits : std::min(tiles_total, 64);
    int min_split = a->num_splits > 0 ? a->num_splits : 1;
    for (int ns = min_split; ns <= max_split; ++ns) {
        const int tiles_per = (tiles_total + ns - 1) / ns;
        const int64_t items = units * ns;
        const int64_t rounds = (items + grid - 1) / grid;
        const double cost = (double)rounds * (tiles_per + 0.75) + (ns > 1 ? 0.25 : 0.0);
        if (cost < best_cost - 1e-9) { best_cost = cost; best = ns; }
    }
    pl.chunk = ((tiles_total + best - 1) / best) * kTT;
    pl.nsplit = (a->seq_len + pl.chunk - 1) / pl.chunk;
    if (pl.nsplit < 1) pl.nsplit = 1;
    return pl;
}

size_t attn_workspace_size(const pkv_codec* c, const pkv_attn_args* a) {
    AttnPlan pl = plan_attn(c, a);
    if (pl.nsplit <= 1) return 0;
    size_t part = (size_t)a->batch * a->q_heads * pl.nsplit * (c->dim + 2) * sizeof(float);
    part = (part + 255) / 256 * 256;
    return part + (size_t)a->batch * a->kv_heads * sizeof(int32_t);
}

template <int CB, int TPL, int G, bool TMA>
static int launch_attn_t(const AttnParams& p, const AttnPlan& pl, cudaStream_t st) {
    auto kern = attn_decode_kernel<CB, TPL, G, TMA>;
    const int threads = TMA ? 160 : 128;
    const size_t smem = pl.L.total;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return PKV_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess || per_sm <= 0)
        return PKV_ERR_CUDA;
    const int grid = (int)std::min<int64_t>(p.num_items, (int64_t)per_sm * num_sms());
    kern<<<grid, threads, smem, st>>>(p);
    return cudaGetLastError() == cudaSuccess ? PKV_OK : PKV_ERR_CUDA;
}

template <int CB, int TPL, int G>
static int launch_attn_g(const AttnParams& p, const AttnPlan& pl, cudaStream_t st) {
    return pl.tma ? launch_attn_t<CB, TPL, G, true>(p, pl, st) : launch_attn_t<CB, TPL, G, false>(p, pl, st);
}

template <int CB, int TPL>
static int launch_attn_tpl(const AttnParams& p, const AttnPlan& pl, cudaStream_t st) {
    switch (pl.G) {
        case 1: return launch_attn_g<CB, TPL, 1>(p, pl, st);
        case 2: return launch_attn_g<CB, TPL, 2>(p, pl, st);
        case 4: return launch_attn_g<CB, TPL, 4>(p, pl, st);
        case 8: return launch_attn_g<CB, TPL, 8>(p, pl, st);
    }
    return PKV_ERR_UNSUPPORTED;
}

template <int CB>
static int launch_attn_cb(const AttnParams& p, const AttnPlan& pl, cudaStream_t st) {
    return pl.TPL == 1 ? launch_attn_tpl<CB, 1>(p, pl, st) : launch_attn_tpl<CB, 2>(p, pl, st);
}

int launch_attn(const pkv_codec* c, const pkv_attn_args* a, void* ws, size_t ws_bytes, cudaStream_t st) {
    AttnPlan pl = plan_attn(c, a);
    if (pl.L.total > 227 * 1024) return PKV_ERR_UNSUPPORTED;
    AttnParams p{};
    p.B = a->batch; p.Hq = a->q_heads; p.Hkv = a->kv_heads; p.S = a->seq_len;
    p.G = a->q_heads / a->kv_heads; p.m = c->dim / 3; p.dim = c->dim;
    p.q = a->q; p.qdt = a->q_dtype; p.q_bs = a->q_batch_stride; p.q_hs = a->q_head_stride;
    p.kc = static_cast<const uint8_t*>(a->k_codes); p.vc = static_cast<const uint8_t*>(a->v_codes);
    p.kv_bs = a->kv_batch_stride; p.kv_hs = a->kv_head_stride;
    p.seq_lens = a->seq_lens;
    p.scale_log2 = a->scale * 1.4426950408889634f;
    p.out = a->out; p.out_bs = a->out_batch_stride; p.out_hs = a->out_head_stride;
    p.nsplit = pl.nsplit; p.chunk = pl.chunk;
    p.partial_only = a->partial_only; p.partial_out = a->partial_out;
    if (pl.nsplit > 1) {
        size_t need = attn_workspace_size(c, a);
        if (!ws || ws_bytes < need) return PKV_ERR_WORKSPACE;
        size_t part = (size_t)a->batch * a->q_heads * pl.nsplit * (c->dim + 2) * sizeof(float);
        part = (part + 255) / 256 * 256;
        p.ws_part = static_cast<float*>(ws);
        p.ws_count = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ws) + part);
    }
    p.R = c->R; p.dec_z = c->dec_z; p.dec_xy = c->dec_xy;
    p.bits_flat = c->bits_r + c->bits_theta;
    p.code_mask = (1 << (c->bits_z + p.bits_flat)) - 1;
    p.flat_mask = (1 << p.bits_flat) - 1;
    p.xy_per_z = c->xy_per_z;
    p.Cz = 1 << c->bits_z;
    p.n_xy = (c->xy_per_z ? p.Cz : 1) << p.bits_flat;
    p.num_items = a->batch * a->kv_heads * pl.nsplit;
    p.stages = pl.stages;
    if (p.num_items == 0) return PKV_OK;
    return a->code_bytes == 1 ? launch_attn_cb<1>(p, pl, st) : launch_attn_cb<2>(p, pl, st);
}

int launch_lse_combine(const pkv_codec* c, const float* parts, int n_parts, int64_t part_stride,
                       int rows, float* out, int64_t out_rs, cudaStream_t st) {
    if (rows == 0) return PKV_OK;
    lse_combine_kernel<<<rows, 128, c->dim * sizeof(float), st>>>(parts, n_parts, part_stride, rows, c->dim,
                                                                   c->R, out, out_rs);
    return cudaGetLastError() == cudaSuccess ? PKV_OK : PKV_ERR_CUDA;
}

}  // namespace pkv
