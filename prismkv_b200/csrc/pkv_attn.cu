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
// Common schedule:
//  * codes: (B, Hkv, S, m) of uint8/uint16, one m-code row per token;
//  * one work item = (b, unit head, split) = a contiguous token range (the
//    unit head is the KV head, or the query head for grouped heads on the
//    one-head kernels); persistent CTAs take items round-robin, or balanced
//    tile ranges (the one-pass LUT kernel);
//  * a producer warp streams code tiles into a shared-memory ring with 1-D
//    TMA bulk copies completing on mbarriers;
//  * splits of one unit write (m, l, o) partials to the workspace; the last
//    CTA to finish (atomic counter) merges them, normalises and applies R
//    once, then resets the counter.
//
// Kernels (plan_attn below picks one per call):
//  * attn_polar_kernel (this file) -- uniform polar (x, y) bins (any z bins,
//    optional BiasTable): two passes per item (K -> scores in shared memory,
//    exact max, then V with fixed weights).  K scores come from per-lane
//    tables indexed by the code fields (one bank per lane: conflict-free), V
//    from a 16-entry (cos, sin) table and the radius index itself.
//  * attn_lut_kernel (this file) -- any codec (learned codebooks): one pass,
//    online softmax, (z, x, y) from full-code LUTs.
//  * attn_mha12_kernel, attn_mha12_stream_kernel (pkv_attn_mha12.cu) -- the
//    12-bit uniform-polar head_dim-96 case, one query head per unit: two
//    passes for sequences of one 4096-token item, one pass beyond.
//  * attn_mha8_kernel (pkv_attn_mha8.cu) -- one-byte uniform-polar codes,
//    head_dim 96, one query head per unit.
//  * attn_tc_kernel (pkv_attn_tc.cu) -- tcgen05 tensor cores for bf16/fp16
//    queries of grouped heads or per-z-bin tables.
//
// Every mbarrier wait is bounded; on expiry the kernel sets the device error
// word, stops issuing copies, drains what it issued and returns.

#include <algorithm>
#include <cmath>

#include "pkv_common.cuh"

namespace pkv {

constexpr float kLn2 = 0.69314718055994530942f;
constexpr float kLog2e = 1.4426950408889634f;

struct AttnParams {
    int B, Hq, Hkv, S, G, m, dim;
    const void* q; int qdt; int64_t q_bs, q_hs;
    const uint8_t* kc; const uint8_t* vc;
    int64_t kv_bs, kv_hs;              // in codes
    const int32_t* seq_lens;
    float scale_log2;
    float* out; int64_t out_bs, out_hs;
    int nsplit, chunk;                 // chunk: tokens per split, multiple of the tile
    int partial_only; float* partial_out;
    float* ws_part; int32_t* ws_count;
    const float* R; const float* dec_z; const float* dec_xy; const float* bias_xy;
    int bits_z, bits_r, bits_t;
    int bits_flat, code_mask, flat_mask, xy_per_z, n_xy, Cz;
    float r_max;
    int num_items, stages;
    // balanced schedule (bal != 0): CTA c streams global tiles [c T / G, (c+1) T / G) of the
    // unit-major tile sequence; segments are cut at unit ends, at every `seg_cap` tiles of a
    // unit and at CTA boundaries.  slots: partial rows kept per (b, q head) in the workspace.
    int bal, tt, tpu, seg_cap, slots;
    int64_t tiles;
    // Hu: work units per batch row -- Hkv, or Hq when every query head is its own unit reading
    // KV head hq / Gq (grouped heads through a one-head kernel; the group's re-reads hit L2)
    int Hu, Gq;
    // split-sequence exchange (pkv_attn_decode_xr) when xr_world > 0: every rank's exchange buffer
    // (partial slots, output rows, counters at the byte offsets below), this rank's index, the
    // units every rank counts, and the bound on the completion wait
    int xr_world, xr_rank, xr_units;
    uint8_t* xr_buf[PKV_XR_MAX_RANKS];
    int64_t xr_out_off, xr_ctl_off;
    uint64_t xr_wait_ns;
};

__host__ __device__ inline int align_up(int x, int a) { return (x + a - 1) / a * a; }

__device__ __forceinline__ float q_load(const void* q, int qdt, int64_t idx) {
    if (qdt == PKV_F32) return __ldg(static_cast<const float*>(q) + idx);
    if (qdt == PKV_BF16) return __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(q) + idx));
    return __half2float(__ldg(static_cast<const __half*>(q) + idx));
}

// One segment of work: tokens [tok0, tok1) of (b, kv head hk).  The unit's
// segments number nseg; this one writes partial slot `split` when nseg > 1.
struct ItemRange { int b, hk, split, tok0, tok1, nseg, kvh; };   // hk: unit head, kvh: its KV head

__device__ __forceinline__ ItemRange item_range(const AttnParams& p, int item) {
    ItemRange r;
    r.nseg = p.nsplit;
    r.split = item % p.nsplit;
    int bh = item / p.nsplit;
    r.hk = bh % p.Hu;
    r.b = bh / p.Hu;
    r.kvh = r.hk / p.Gq;
    int L = p.seq_lens ? min(max(p.seq_lens[r.b], 0), p.S) : p.S;
    r.tok0 = r.split * p.chunk;
    r.tok1 = min(L, r.tok0 + p.chunk);
    if (r.tok1 < r.tok0) r.tok1 = r.tok0;
    return r;
}

// Cut points strictly inside unit tiles [a, b): chunk cuts a + k seg_cap and the
// CTA boundaries floor(c T / G).  slot = cuts in (a, t]; nseg = 1 + cuts in (a, b).
__device__ inline void balanced_slot(const AttnParams& p, int64_t a, int64_t b, int64_t t, int G, int& slot,
                                     int& nseg) {
    const int64_t T = p.tiles, cap = p.seg_cap;
    int in_unit = (int)((b - a - 1) / cap), upto_t = (int)((t - a) / cap);
    for (int64_t c = ((a + 1) * G + T - 1) / T; c < G; ++c) {
        const int64_t cut = c * T / G;
        if (cut >= b) break;
        if ((cut - a) % cap != 0) {
            ++in_unit;
            if (cut <= t) ++upto_t;
        }
    }
    slot = upto_t;
    nseg = 1 + in_unit;
}

// Work cursor shared by the producer and the consumers of a CTA: both walk the
// same segment sequence.  Round-robin items (bal == 0) or the balanced tile range.
struct WorkCursor { int64_t t, t_end; int item; };

__device__ __forceinline__ WorkCursor work_begin(const AttnParams& p) {
    WorkCursor c;
    c.item = blockIdx.x;
    c.t = (int64_t)blockIdx.x * p.tiles / gridDim.x;
    c.t_end = (int64_t)(blockIdx.x + 1) * p.tiles / gridDim.x;
    return c;
}

// BAL = false compiles the balanced branch out (kernels the planner never balances).
template <bool BAL>
__device__ inline bool work_next(const AttnParams& p, WorkCursor& c, ItemRange& r) {
    if (!BAL || !p.bal) {
        if (c.item >= p.num_items) return false;
        r = item_range(p, c.item);
        c.item += gridDim.x;
        return true;
    }
    if (c.t >= c.t_end) return false;
    const int64_t u = c.t / p.tpu, a = u * p.tpu, b = a + p.tpu;
    const int64_t cb = a + ((c.t - a) / p.seg_cap + 1) * p.seg_cap;
    const int64_t e = min(c.t_end, min(b, cb));
    r.hk = (int)(u % p.Hu);
    r.b = (int)(u / p.Hu);
    r.kvh = r.hk / p.Gq;
    r.tok0 = (int)(c.t - a) * p.tt;
    r.tok1 = min(p.S, (int)(e - a) * p.tt);
    balanced_slot(p, a, b, c.t, gridDim.x, r.split, r.nseg);
    c.t = e;
    return true;
}

// transpose-reduce: on entry each lane holds v[0..31]; on exit v[0] of lane l
// holds the sum over all lanes of their v[l].
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

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    // d = a * b + c on two fp32 lanes (sm_100 paired FMA), operands packed in registers
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// rotated, scaled query of every head of the group -> sQ[G][dim]:
// sQ[g][k] = scale*log2(e) * sum_i q[g][i] R[k][i].  The raw query is staged in
// shared memory (sQraw, G*dim floats); one thread per output row k issues all
// loads of row k before the multiply-adds, so a rotation costs one memory
// round trip.  Rp: R with row pitch `pitch` (global or shared).
template <int G>
__device__ __forceinline__ void rotate_query(const AttnParams& p, const ItemRange& r, const float* Rp, int pitch,
                                             float* sQ, float* sQraw, int tid, int nthr) {
    const int dim = p.dim;
    for (int idx = tid; idx < G * dim; idx += nthr) {
        const int g = idx / dim, i = idx % dim;
        float v = 0.f;
        if (g < p.G) {
            const int hq = r.hk * p.G + g;
            v = q_load(p.q, p.qdt, (int64_t)r.b * p.q_bs + (int64_t)hq * p.q_hs + i);
        }
        sQraw[idx] = v;
    }
    named_bar_sync(1, nthr);
    for (int k = tid; k < dim; k += nthr) {
        const float* row = Rp + k * pitch;
        float acc[G];
        #pragma unroll
        for (int g = 0; g < G; ++g) acc[g] = 0.f;
        for (int i0 = 0; i0 < dim; i0 += 32) {
            float rv[32];
            #pragma unroll
            for (int u = 0; u < 32; ++u) rv[u] = (i0 + u < dim) ? row[i0 + u] : 0.f;
            #pragma unroll
            for (int g = 0; g < G; ++g)
                #pragma unroll
                for (int u = 0; u < 32; ++u)
                    if (i0 + u < dim) acc[g] = fmaf(sQraw[g * dim + i0 + u], rv[u], acc[g]);
        }
        #pragma unroll
        for (int g = 0; g < G; ++g) sQ[g * dim + k] = acc[g] * p.scale_log2;
    }
}

// ---------------------------------------------------------------------------
// split-sequence exchange (the peers are other GPUs, reached through CUDA-IPC peer memory).
// Protocol with the flag in the word: every partial value travels as one 8-byte store of (value,
// flag), flag = epoch + 1, and a naturally aligned 8-byte access is single-copy atomic, so a
// reader that sees the flag sees the value -- no fences, no counters.  The epoch counts this
// rank's calls (advanced by the call's last CTA); the slots alternate by its parity, so a rank one
// call ahead never overwrites what a slower rank still reads (it cannot get two calls ahead: its
// next call needs the slower rank's partials of that call).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* ptr, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" :: "l"(ptr), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* ptr) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(ptr) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// This call's epoch (control word 0 of this rank's buffer; it changes only after every CTA of
// the call is done).
__device__ __forceinline__ uint32_t xr_epoch(const AttnParams& p) {
    return *reinterpret_cast<const volatile uint32_t*>(p.xr_buf[p.xr_rank] + p.xr_ctl_off);
}

// Word k of the partial row `row` from rank `src` in rank `dst`'s buffer, slot parity `par`.
__device__ __forceinline__ uint64_t* xr_word(const AttnParams& p, int dst, uint32_t par, int src, int64_t row, int k) {
    return reinterpret_cast<uint64_t*>(p.xr_buf[dst]) +
           ((((int64_t)par * p.xr_world + src) * p.B * p.Hq + row) * (p.dim + 2) + k);
}

// Output element (query head g of the item's unit, dim i): the caller's output, or in exchange
// mode this rank's output rows (every rank merges its own copy).
__device__ __forceinline__ void store_out(const AttnParams& p, const ItemRange& r, int g, int i, float v) {
    const int hq = r.hk * p.G + g;
    if (p.xr_world > 0) {
        const int64_t off = p.xr_out_off + (((int64_t)r.b * p.Hq + hq) * p.dim + i) * 4;
        *reinterpret_cast<float*>(p.xr_buf[p.xr_rank] + off) = v;
    } else {
        p.out[(int64_t)r.b * p.out_bs + (int64_t)hq * p.out_hs + i] = v;
    }
}

// Exchange mode: element k of this rank's final partial row of query head g ([m (log2 units), l,
// o_rot]) into slot xr_rank of every rank's buffer, flagged with this call's epoch.
__device__ __forceinline__ void xr_publish(const AttnParams& p, const ItemRange& r, int g, int k, float val,
                                           uint32_t epoch) {
    const int64_t row = (int64_t)r.b * p.Hq + r.hk * p.G + g;
    const uint64_t w = ((uint64_t)(epoch + 1u) << 32) | (uint64_t)__float_as_uint(val);
    for (int s = 0; s < p.xr_world; ++s) st_relaxed_sys_u64(xr_word(p, s, epoch & 1u, p.xr_rank, row, k), w);
}

// The value of a flagged word once its flag is this call's, bounded by xr_wait_ns from t0 (or
// given up at once when the device error word is already set); on expiry the error word is set
// and 0 returned.
__device__ __forceinline__ float xr_take(const uint64_t* ptr, uint32_t flag, uint64_t t0, uint64_t limit) {
    for (;;) {
        const uint64_t w = ld_relaxed_sys_u64(ptr);
        if ((uint32_t)(w >> 32) == flag) return __uint_as_float((uint32_t)w);
        if (*reinterpret_cast<volatile int32_t*>(&g_device_error) != 0) return 0.f;
        if (global_ns() - t0 > limit) {
            flag_error(kErrPeerWait);
            return 0.f;
        }
        __nanosleep(64);
    }
}

// out rows of the item's unit = (sFin rows) @ R, through store_out.  With parts > 1, up to
// max_parts threads share an output, each summing a slice of k with two chains; sO (at least
// max_parts * G * dim floats, dead by now) holds their partial sums.  With one part, each thread
// batches 48 loads of R ahead of its FMAs (two L2 round trips for head_dim 96 when R is global).
__device__ void rotate_out(const AttnParams& p, const ItemRange& r, float* sO, const float* sFin, const float* Rp,
                           int pitch, int tid, int nthr, int max_parts) {
    const int dim = p.dim, greal = p.G;
    named_bar_sync(1, nthr);
    const int gd = greal * dim;
    const int parts = max(1, min(max_parts, nthr / gd));
    if (parts == 1) {
        for (int idx = tid; idx < gd; idx += nthr) {
            const int g = idx / dim, i = idx % dim;
            float v = 0.f;
            for (int k0 = 0; k0 < dim; k0 += 48) {
                float rv[48];
                #pragma unroll
                for (int u = 0; u < 48; ++u) rv[u] = (k0 + u < dim) ? Rp[(k0 + u) * pitch + i] : 0.f;
                #pragma unroll
                for (int u = 0; u < 48; ++u)
                    if (k0 + u < dim) v = fmaf(sFin[g * dim + k0 + u], rv[u], v);
            }
            store_out(p, r, g, i, v);
        }
        return;
    }
    const int klen = (dim + parts - 1) / parts;
    for (int idx = tid; idx < gd * parts; idx += nthr) {
        const int part = idx / gd, gi = idx % gd, g = gi / dim, i = gi % dim;
        const int k1 = min(dim, (part + 1) * klen);
        const float* f = sFin + g * dim;
        float v0 = 0.f, v1 = 0.f;
        int k = part * klen;
        #pragma unroll 8
        for (; k + 1 < k1; k += 2) {
            v0 = fmaf(f[k], Rp[k * pitch + i], v0);
            v1 = fmaf(f[k + 1], Rp[(k + 1) * pitch + i], v1);
        }
        if (k < k1) v0 = fmaf(f[k], Rp[k * pitch + i], v0);
        sO[idx] = v0 + v1;
    }
    named_bar_sync(1, nthr);
    for (int gi = tid; gi < gd; gi += nthr) {
        float v = 0.f;
        for (int part = 0; part < parts; ++part) v += sO[part * gd + gi];
        store_out(p, r, gi / dim, gi % dim, v);
    }
}

// Exchange mode: wait for every rank's partial rows of the unit in this rank's buffer (flag =
// this call's epoch + 1), merge them (log-sum-exp), apply R once and store this rank's output rows.
__device__ void xr_merge_unit(const AttnParams& p, const ItemRange& r, float* sO, float* sFin, const float* Rp,
                              int pitch, int tid, int nthr, int max_parts) {
    const int dim = p.dim, greal = p.G;
    named_bar_sync(1, nthr);
    const uint32_t epoch = xr_epoch(p), flag = epoch + 1u, par = epoch & 1u;
    const uint64_t t0 = global_ns();
    for (int idx = tid; idx < greal * dim; idx += nthr) {
        const int g = idx / dim, k = idx % dim;
        const int64_t row = (int64_t)r.b * p.Hq + r.hk * greal + g;
        float ms[PKV_XR_MAX_RANKS], ls[PKV_XR_MAX_RANKS], os[PKV_XR_MAX_RANKS];
        float M = -INFINITY;
        #pragma unroll
        for (int s = 0; s < PKV_XR_MAX_RANKS; ++s) {
            if (s >= p.xr_world) break;
            ms[s] = xr_take(xr_word(p, p.xr_rank, par, s, row, 0), flag, t0, p.xr_wait_ns);
            ls[s] = xr_take(xr_word(p, p.xr_rank, par, s, row, 1), flag, t0, p.xr_wait_ns);
            os[s] = xr_take(xr_word(p, p.xr_rank, par, s, row, 2 + k), flag, t0, p.xr_wait_ns);
            M = fmaxf(M, ms[s]);
        }
        float v = 0.f, l = 0.f;
        #pragma unroll
        for (int s = 0; s < PKV_XR_MAX_RANKS; ++s) {
            if (s >= p.xr_world) break;
            const float f = (ms[s] == -INFINITY) ? 0.f : fast_exp2(ms[s] - M);
            l = fmaf(ls[s], f, l);
            v = fmaf(os[s], f, v);
        }
        sFin[g * dim + k] = (l > 0.f) ? v / l : 0.f;
    }
    rotate_out(p, r, sO, sFin, Rp, pitch, tid, nthr, max_parts);
}

// Exchange mode, once per CTA after its last item (every kernel's tail): merge the units assigned
// to this CTA (u = blockIdx.x, + gridDim.x, ...) into this rank's output rows; then the call's
// last CTA advances the epoch (every CTA has merged its units by then; the next call, stream-
// ordered, reads the new epoch).  A CTA waits for partials only after it has published all of its
// own, so no two CTAs of any ranks can wait on each other.  sO / sFin / R as for finish_item.
__device__ void xr_finish_call(const AttnParams& p, float* sO, float* sFin, const float* Rp, int pitch, int tid,
                               int nthr, int max_parts) {
    if (p.xr_world <= 0) return;
    for (int u = blockIdx.x; u < p.xr_units; u += gridDim.x) {
        ItemRange r{};
        r.b = u / p.Hu;
        r.hk = u % p.Hu;
        xr_merge_unit(p, r, sO, sFin, Rp, pitch, tid, nthr, max_parts);
        named_bar_sync(1, nthr);                      // sO / sFin free for the next unit
    }
    named_bar_sync(1, nthr);
    if (tid != 0) return;
    uint32_t* ctl = reinterpret_cast<uint32_t*>(p.xr_buf[p.xr_rank] + p.xr_ctl_off);
    __threadfence();
    if (atomicAdd(ctl + 1, 1u) != gridDim.x - 1) return;
    *reinterpret_cast<volatile uint32_t*>(ctl + 1) = 0u;
    *reinterpret_cast<volatile uint32_t*>(ctl) = ctl[0] + 1u;
    __threadfence();
}

// Per-item epilogue shared by the kernels.  Inputs in shared memory, per head g < greal: sM[g]
// (running max, log2 units), sL[g], sO[g*dim + k] (unnormalised rotated-space output).  Writes
// the partial row, or merges splits and writes out = (o / l) @ R, or (exchange mode) publishes
// the unit's partial rows to every rank and takes part in the cross-rank merge.  All `nthr`
// consumer threads call it; barrier id 1.
__device__ void finish_item(const AttnParams& p, const ItemRange& r, const float* sM, const float* sL,
                            float* sO, float* sFin, int* sflag, const float* Rp, int pitch, int tid,
                            int nthr, int max_parts) {
    const int dim = p.dim, greal = p.G;
    const bool single = (r.nseg == 1);
    const bool xr = p.xr_world > 0;
    const uint32_t epoch = xr ? xr_epoch(p) : 0u;
    bool finalize = single && !p.partial_only && !xr;
    bool arrive = single && xr;
    for (int idx = tid; idx < greal * (dim + 2); idx += nthr) {
        const int g = idx / (dim + 2), k = idx % (dim + 2);
        const float M = sM[g], L = sL[g];
        const int hq = r.hk * greal + g;
        if (finalize) {
            if (k >= 2) sFin[g * dim + (k - 2)] = (L > 0.f) ? sO[g * dim + (k - 2)] / L : 0.f;
        } else {
            const float val = (k == 0) ? M : (k == 1 ? L : sO[g * dim + (k - 2)]);
            if (!single) {
                float* dst = p.ws_part + (((int64_t)r.b * p.Hq + hq) * p.slots + r.split) * (dim + 2);
                dst[k] = val;
            } else if (xr) {
                xr_publish(p, r, g, k, val, epoch);
            } else {
                float* dst = p.partial_out + ((int64_t)r.b * p.Hq + hq) * (dim + 2);
                dst[k] = (k == 0) ? (M == -INFINITY ? -INFINITY : M * kLn2) : val;
            }
        }
    }
    if (!single) {
        __threadfence();
        named_bar_sync(1, nthr);
        if (tid == 0) {
            int32_t* cnt = p.ws_count + (r.b * p.Hu + r.hk);
            const int prev = atomicAdd(cnt, 1);
            const int last = (prev == r.nseg - 1);
            if (last) { __threadfence(); atomicExch(cnt, 0); }
            sflag[0] = last;
        }
        named_bar_sync(1, nthr);
        if (sflag[0]) {
            for (int idx = tid; idx < greal * (dim + 2); idx += nthr) {
                const int g = idx / (dim + 2), k = idx % (dim + 2);
                const int hq = r.hk * greal + g;
                const float* src = p.ws_part + ((int64_t)r.b * p.Hq + hq) * p.slots * (dim + 2);
                float M = -INFINITY;
                for (int sp = 0; sp < r.nseg; ++sp) M = fmaxf(M, __ldcg(src + sp * (dim + 2)));
                float v = 0.f, lsw = 0.f;
                for (int sp = 0; sp < r.nseg; ++sp) {
                    const float ms = __ldcg(src + sp * (dim + 2));
                    const float f = (ms == -INFINITY) ? 0.f : fast_exp2(ms - M);
                    lsw = fmaf(__ldcg(src + sp * (dim + 2) + 1), f, lsw);
                    if (k >= 2) v = fmaf(__ldcg(src + sp * (dim + 2) + k), f, v);
                }
                if (xr) {
                    xr_publish(p, r, g, k, (k == 0) ? M : (k == 1 ? lsw : v), epoch);
                } else if (p.partial_only) {
                    float* dst = p.partial_out + ((int64_t)r.b * p.Hq + hq) * (dim + 2);
                    dst[k] = (k == 0) ? (M == -INFINITY ? -INFINITY : M * kLn2) : (k == 1 ? lsw : v);
                } else if (k >= 2) {
                    sFin[g * dim + (k - 2)] = (lsw > 0.f) ? v / lsw : 0.f;
                }
            }
            // Clear the consumed partials: a workspace shared by calls of other shapes puts its
            // counters at other offsets, so every byte must be zero again after each call.
            named_bar_sync(1, nthr);
            for (int g = 0; g < greal; ++g) {
                float* rows = p.ws_part + ((int64_t)r.b * p.Hq + (int64_t)r.hk * greal + g) * p.slots * (dim + 2);
                for (int k = tid; k < r.nseg * (dim + 2); k += nthr) rows[k] = 0.f;
            }
            finalize = !p.partial_only && !xr;
            arrive = xr;
        }
    }
    (void)arrive;                                     // exchange: merged at the CTA's end (xr_finish_call)
    if (finalize) rotate_out(p, r, sO, sFin, Rp, pitch, tid, nthr, max_parts);
    // the next item may overwrite sFin / sO / sflag only after every thread is done with them
    named_bar_sync(1, nthr);
}

// Producer loop: for every item, `passes` sweeps over its token range (K then V
// for the two-pass kernel; K+V tiles together for the one-pass kernel).
template <int TT, bool KV_TOGETHER, bool BAL>
__device__ void produce(const AttnParams& p, uint8_t* stage_base, int stage_bytes, uint64_t* full,
                        uint64_t* empty, int ncons_warps, int code_bytes) {
    const uint32_t row_bytes = (uint32_t)(p.m * code_bytes);
    int seq = 0;
    bool ok = true;
    WorkCursor wc = work_begin(p);
    ItemRange r;
    while (ok && work_next<BAL>(p, wc, r)) {
        const int64_t base = ((int64_t)r.b * p.kv_bs + (int64_t)r.kvh * p.kv_hs) * code_bytes;
        for (int pass = 0; pass < (KV_TOGETHER ? 1 : 2) && ok; ++pass) {
            for (int t0 = r.tok0; t0 < r.tok1; t0 += TT, ++seq) {
                const int s = seq % p.stages;
                const int use = seq / p.stages;
                if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, kErrWaitEmpty)) { ok = false; break; }
                const int nt = min(TT, r.tok1 - t0);
                const uint32_t bytes = (uint32_t)nt * row_bytes;
                uint8_t* dst = stage_base + s * stage_bytes;
                const int64_t off = base + (int64_t)t0 * row_bytes;
                if (KV_TOGETHER) {
                    mbar_arrive_expect_tx(&full[s], 2 * bytes);
                    bulk_g2s(dst, p.kc + off, bytes, &full[s]);
                    bulk_g2s(dst + TT * row_bytes, p.vc + off, bytes, &full[s]);
                } else {
                    mbar_arrive_expect_tx(&full[s], bytes);
                    bulk_g2s(dst, (pass == 0 ? p.kc : p.vc) + off, bytes, &full[s]);
                }
            }
        }
    }
    const int issued = seq;                           // drain before the CTA may exit
    for (int q = max(0, issued - p.stages); q < issued; ++q)
        mbar_wait(&full[q % p.stages], (q / p.stages) & 1, kErrWaitDrain);
}

// ===========================================================================
// attn_polar_kernel
// ===========================================================================
constexpr int kPW = 8;            // consumer warps
constexpr int kPTT = 256;         // tokens per tile (32 per consumer warp)
constexpr int kPChunk = 4096;     // score entries kept per item (all heads of the group)

struct PolarLayout {
    int stage_bytes, stages, kxy, ct, cz, chunk;
    int off_stage, off_kt, off_kz, off_vz, off_cs, off_vb, off_q, off_s, off_red, off_acc, off_fin, off_misc,
        off_bar, total;
};

__host__ __device__ inline PolarLayout polar_layout(int m, int cb, int dim, int G, int bits_z, int bits_r,
                                                    int bits_t, int stages) {
    PolarLayout L;
    L.stages = stages;
    L.kxy = 1 << (bits_r + bits_t);
    L.ct = 1 << bits_t;
    L.cz = 1 << bits_z;
    L.chunk = kPChunk / G;
    L.stage_bytes = kPTT * m * cb;
    int o = 0;
    L.off_stage = o; o += stages * L.stage_bytes; o = align_up(o, 128);
    L.off_kt = o; o += (G == 1 ? L.kxy : G * L.ct) * 32 * 4; o = align_up(o, 128);     // per-lane K tables
    L.off_kz = o; o += G * L.cz * 32 * 4; o = align_up(o, 128);
    L.off_vz = o; o += L.cz * 4; o = align_up(o, 128);
    L.off_cs = o; o += L.ct * 8; o = align_up(o, 128);
    L.off_vb = o; o += L.cz * 8; o = align_up(o, 16);
    L.off_q = o; o += G * dim * 4; o = align_up(o, 16);
    L.off_s = o; o += G * L.chunk * 4; o = align_up(o, 16);
    L.off_red = o; o += kPW * G * 4 * 2; o = align_up(o, 16);
    L.off_acc = o; o += kPW * G * dim * 4; o = align_up(o, 16);
    L.off_fin = o; o += G * dim * 4; o = align_up(o, 16);
    L.off_misc = o; o += (2 * G + 4) * 4; o = align_up(o, 16);
    L.off_bar = o; o += 2 * stages * 8;
    L.total = o;
    return L;
}

template <int CB, int G, bool BIAS>
__global__ void __launch_bounds__(kPW * 32 + 32, 2) attn_polar_kernel(AttnParams p) {
    using CT = typename Code<CB>::T;
    constexpr int TB = 32 / G;                     // tokens per transpose block
    extern __shared__ __align__(128) uint8_t polar_smem[];
    uint8_t* smem = polar_smem;
    const PolarLayout L = polar_layout(p.m, CB, p.dim, G, p.bits_z, p.bits_r, p.bits_t, p.stages);
    float* kT = reinterpret_cast<float*>(smem + L.off_kt);     // G==1: [kxy][32]; else [G][ct][32]
    float* kZ = reinterpret_cast<float*>(smem + L.off_kz);     // [G][cz][32]
    float* vZ = reinterpret_cast<float*>(smem + L.off_vz);     // [cz]
    float2* vCS = reinterpret_cast<float2*>(smem + L.off_cs);  // [ct]  dr*2^-bt*(cos, sin)
    float2* vB = reinterpret_cast<float2*>(smem + L.off_vb);   // [cz]  -(bias x, bias y)
    float* sQ = reinterpret_cast<float*>(smem + L.off_q);      // [G][dim]
    float* sS = reinterpret_cast<float*>(smem + L.off_s);      // [G][chunk] scores -> weights
    float* sRed = reinterpret_cast<float*>(smem + L.off_red);  // [kPW][G] x2
    float* sAcc = reinterpret_cast<float*>(smem + L.off_acc);  // [kPW][G][dim]
    float* sFin = reinterpret_cast<float*>(smem + L.off_fin);
    float* sM = reinterpret_cast<float*>(smem + L.off_misc);   // [G]
    float* sL = sM + G;                                        // [G]
    int* sflag = reinterpret_cast<int*>(sL + G);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.off_bar);
    uint64_t* empty = full + p.stages;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int dim = p.dim, m = p.m;
    const int bf = p.bits_flat, bt = p.bits_t;
    const uint32_t tmask = (1u << bt) - 1u, fmask = (1u << bf) - 1u;
    const uint32_t rmask = ((1u << p.bits_r) - 1u) << bt;
    const uint32_t cmask = (uint32_t)p.code_mask;     // codes index the tables only after masking
    const float dr = p.r_max / (float)((1 << p.bits_r) - 1);

    // ---- query-independent tables ---------------------------------------
    for (int i = tid; i < L.cz; i += blockDim.x) {
        vZ[i] = __ldg(p.dec_z + i);
        if (BIAS) vB[i] = make_float2(-__ldg(p.bias_xy + 2 * i), -__ldg(p.bias_xy + 2 * i + 1));
    }
    for (int i = tid; i < L.ct; i += blockDim.x) {
        // theta_i = i / (C - 1) * 2 pi - pi (stacked_plane.py:307); scaled so that
        // (i_r << bits_theta) * vCS = r(i_r) * (cos, sin)
        const float th = (float)i / (float)(L.ct - 1) * 6.283185307179586f - 3.141592653589793f;
        const float sc = dr * exp2f((float)-bt);
        vCS[i] = make_float2(cosf(th) * sc, sinf(th) * sc);
    }
    if (tid == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kPW);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kPW) {
        if (lane == 0) produce<kPTT, false, false>(p, smem + L.off_stage, L.stage_bytes, full, empty, kPW, CB);
        return;
    }

    const int nthr = kPW * 32;
    const int myh = lane / TB, myt = lane % TB;
    int seq = 0;
    bool alive = true;
    WorkCursor wc = work_begin(p);
    ItemRange r;
    while (work_next<false>(p, wc, r)) {
        const int ntok = r.tok1 - r.tok0;
        const int ntiles = (ntok + kPTT - 1) / kPTT;
        rotate_query<G>(p, r, p.R, dim, sQ, sFin, tid, nthr);
        named_bar_sync(1, nthr);
        // ---- query tables: one column per lane (bank = lane) ----------------
        if (G == 1) {
            for (int idx = tid; idx < L.kxy * 32; idx += nthr) {
                const int e = idx >> 5, j = idx & 31;
                float v = 0.f;
                if (j < m) {
                    const float fr = (float)((e >> bt) << bt);
                    const float2 cs = vCS[e & tmask];
                    v = fr * (sQ[3 * j + 1] * cs.x + sQ[3 * j + 2] * cs.y);
                }
                kT[idx] = v;
            }
        } else {
            for (int idx = tid; idx < G * L.ct * 32; idx += nthr) {
                const int g = idx / (L.ct * 32), e = (idx >> 5) % L.ct, j = idx & 31;
                float v = 0.f;
                if (j < m) {
                    const float2 cs = vCS[e];
                    v = sQ[g * dim + 3 * j + 1] * cs.x + sQ[g * dim + 3 * j + 2] * cs.y;
                }
                kT[idx] = v;
            }
        }
        for (int idx = tid; idx < G * L.cz * 32; idx += nthr) {
            const int g = idx / (L.cz * 32), e = (idx >> 5) % L.cz, j = idx & 31;
            float v = 0.f;
            if (j < m) {
                v = sQ[g * dim + 3 * j] * vZ[e];
                if (BIAS) v += sQ[g * dim + 3 * j + 1] * vB[e].x + sQ[g * dim + 3 * j + 2] * vB[e].y;
            }
            kZ[idx] = v;
        }
        named_bar_sync(1, nthr);

        // ---- pass 1: K codes -> scores --------------------------------------
        float mx = -INFINITY;                      // this lane's head: myh
        for (int tile = 0; tile < ntiles; ++tile, ++seq) {
            const int s = seq % p.stages;
            if (alive && !mbar_wait(&full[s], (seq / p.stages) & 1, kErrWaitFull)) alive = false;
            const CT* Kt = reinterpret_cast<const CT*>(smem + L.off_stage + s * L.stage_bytes);
            const int nt = min(kPTT, ntok - tile * kPTT);
            if (alive && warp * 32 < nt) {
                #pragma unroll 1
                for (int blk = 0; blk < G; ++blk) {
                    const int tl0 = warp * 32 + blk * TB;
                    float ps[32];
                    #pragma unroll
                    for (int t = 0; t < TB; ++t) {
                        const uint32_t c = (lane < m) ? ((uint32_t)Kt[(tl0 + t) * m + lane] & cmask) : 0u;
                        if (G == 1) {
                            ps[t] = kT[((c & fmask) << 5) + lane] + kZ[((c >> bf) << 5) + lane];
                        } else {
                            const float fr = __int_as_float((c & rmask) | 0x4B000000u) - 8388608.f;
                            const uint32_t ti = ((c & tmask) << 5) + lane, zi = ((c >> bf) << 5) + lane;
                            #pragma unroll
                            for (int g = 0; g < G; ++g)
                                ps[g * TB + t] = fmaf(fr, kT[g * L.ct * 32 + ti], kZ[g * L.cz * 32 + zi]);
                        }
                    }
                    transpose_reduce32(ps, lane);
                    const int tok = tl0 + myt;
                    if (tok < nt && myh < p.G) {
                        sS[myh * L.chunk + tile * kPTT + tok] = ps[0];
                        mx = fmaxf(mx, ps[0]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // ---- exact max per head, weights, l -----------------------------------
        #pragma unroll
        for (int off = TB / 2; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        if (myt == 0) sRed[warp * G + myh] = mx;
        named_bar_sync(1, nthr);
        if (tid < G) {
            float M = -INFINITY;
            for (int w = 0; w < kPW; ++w) M = fmaxf(M, sRed[w * G + tid]);
            sM[tid] = M;
        }
        named_bar_sync(1, nthr);
        {
            const int span = ntiles * kPTT;
            float lp[G];
            #pragma unroll
            for (int g = 0; g < G; ++g) {
                lp[g] = 0.f;
                const float M = sM[g];
                for (int t = tid; t < span; t += nthr) {
                    const float pv = (t < ntok && M != -INFINITY) ? fast_exp2(sS[g * L.chunk + t] - M) : 0.f;
                    sS[g * L.chunk + t] = pv;
                    lp[g] += pv;
                }
                #pragma unroll
                for (int off = 16; off >= 1; off >>= 1) lp[g] += __shfl_xor_sync(0xffffffffu, lp[g], off);
                if (lane == 0) sRed[kPW * G + warp * G + g] = lp[g];
            }
        }
        named_bar_sync(1, nthr);
        if (tid < G) {
            float l = 0.f;
            for (int w = 0; w < kPW; ++w) l += sRed[kPW * G + w * G + tid];
            sL[tid] = l;
        }

        // ---- pass 2: V codes, fixed weights -----------------------------------
        float2 axy[G];
        float az[G];
        #pragma unroll
        for (int g = 0; g < G; ++g) { axy[g] = make_float2(0.f, 0.f); az[g] = 0.f; }
        for (int tile = 0; tile < ntiles; ++tile, ++seq) {
            const int s = seq % p.stages;
            if (alive && !mbar_wait(&full[s], (seq / p.stages) & 1, kErrWaitFull)) alive = false;
            const CT* Vt = reinterpret_cast<const CT*>(smem + L.off_stage + s * L.stage_bytes);
            const int nt = min(kPTT, ntok - tile * kPTT);
            if (alive && warp * 32 < nt && lane < m) {
                const float* pw = sS + tile * kPTT + warp * 32;
                #pragma unroll 8
                for (int t = 0; t < 32; ++t) {
                    const uint32_t c = (uint32_t)Vt[(warp * 32 + t) * m + lane] & cmask;
                    const float z = vZ[c >> bf];
                    const float2 cs = vCS[c & tmask];
                    const float fr = __int_as_float((c & rmask) | 0x4B000000u) - 8388608.f;
                    float2 b2;
                    if (BIAS) b2 = vB[c >> bf];
                    #pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float pg = pw[g * L.chunk + t];
                        az[g] = fmaf(pg, z, az[g]);
                        const float w = pg * fr;
                        axy[g] = ffma2(make_float2(w, w), cs, axy[g]);
                        if (BIAS) axy[g] = ffma2(make_float2(pg, pg), b2, axy[g]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // ---- merge warps --------------------------------------------------------
        if (lane < m) {
            #pragma unroll
            for (int g = 0; g < G; ++g) {
                float* o = sAcc + (warp * G + g) * dim + 3 * lane;
                o[0] = az[g]; o[1] = axy[g].x; o[2] = axy[g].y;
            }
        }
        named_bar_sync(1, nthr);
        for (int idx = tid; idx < G * dim; idx += nthr) {
            float v = 0.f;
            #pragma unroll
            for (int w = 0; w < kPW; ++w) v += sAcc[w * G * dim + idx];
            sAcc[idx] = v;                      // warp 0's slot now holds the sum
        }
        named_bar_sync(1, nthr);
        finish_item(p, r, sM, sL, sAcc, sFin, sflag, p.R, dim, tid, nthr, 4);
    }
    xr_finish_call(p, sAcc, sFin, p.R, dim, tid, nthr, 4);
}

// ---------------------------------------------------------------------------
// paired fp32 arithmetic and shared-memory loads by address (the one-head kernels)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

__device__ __forceinline__ float lds_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ float2 lds_f32x2(uint32_t addr) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
    return v;
}

// ===========================================================================
// attn_lut_kernel (any codec)
// ===========================================================================
constexpr int kLW = 4;             // consumer warps
constexpr int kLTT = 128;          // tokens per tile (32 per consumer warp)

struct LutLayout {
    int stage_bytes, stages;
    int off_stage, off_R, off_xy, off_z, off_q, off_cm, off_cl, off_co, off_fin, off_misc, off_bar, total;
};

__host__ __device__ inline LutLayout lut_layout(int m, int cb, int dim, int G, int n_xy, int Cz, int stages) {
    LutLayout L;
    L.stages = stages;
    L.stage_bytes = 2 * kLTT * m * cb;
    int o = 0;
    L.off_stage = o; o += stages * L.stage_bytes; o = align_up(o, 16);
    L.off_R = o; o += dim * (dim + 1) * 4; o = align_up(o, 16);
    L.off_xy = o; o += n_xy * 8; o = align_up(o, 16);
    L.off_z = o; o += Cz * 4; o = align_up(o, 16);
    L.off_q = o; o += G * dim * 4; o = align_up(o, 16);
    L.off_cm = o; o += kLW * G * 4;
    L.off_cl = o; o += kLW * G * 4; o = align_up(o, 16);
    L.off_co = o; o += kLW * G * dim * 4; o = align_up(o, 16);
    L.off_fin = o; o += G * dim * 4; o = align_up(o, 16);
    L.off_misc = o; o += (3 * G + 4) * 4 + G * dim * 4; o = align_up(o, 16);
    L.off_bar = o; o += 2 * stages * 8;
    L.total = o;
    return L;
}

template <int CB, int TPL, int G, bool TMA>
__global__ void __launch_bounds__(TMA ? kLW * 32 + 32 : kLW * 32) attn_lut_kernel(AttnParams p) {
    using CT = typename Code<CB>::T;
    constexpr int TB = 32 / G;
    extern __shared__ __align__(128) uint8_t lut_smem[];
    uint8_t* smem = lut_smem;
    const LutLayout L = lut_layout(p.m, CB, p.dim, G, p.n_xy, p.Cz, p.stages);
    float* sR = reinterpret_cast<float*>(smem + L.off_R);          // R[k][i], pitch dim+1
    const float2* sXY = reinterpret_cast<const float2*>(smem + L.off_xy);
    const float* sZ = reinterpret_cast<const float*>(smem + L.off_z);
    float* sQ = reinterpret_cast<float*>(smem + L.off_q);
    float* sCm = reinterpret_cast<float*>(smem + L.off_cm);
    float* sCl = reinterpret_cast<float*>(smem + L.off_cl);
    float* sCo = reinterpret_cast<float*>(smem + L.off_co);
    float* sFin = reinterpret_cast<float*>(smem + L.off_fin);
    float* sM = reinterpret_cast<float*>(smem + L.off_misc);
    float* sL = sM + G;
    int* sflag = reinterpret_cast<int*>(sL + G);
    float* sO = reinterpret_cast<float*>(smem + L.off_misc) + 3 * G + 4;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.off_bar);
    uint64_t* empty = full + p.stages;

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int dim = p.dim, m = p.m, pitch = dim + 1;

    for (int idx = tid; idx < dim * dim; idx += blockDim.x) {
        int k = idx / dim, i = idx % dim;
        sR[k * pitch + i] = __ldg(p.R + idx);
    }
    {
        float2* xy = reinterpret_cast<float2*>(smem + L.off_xy);
        const float2* g = reinterpret_cast<const float2*>(p.dec_xy);
        for (int idx = tid; idx < p.n_xy; idx += blockDim.x) xy[idx] = __ldg(g + idx);
        float* z = reinterpret_cast<float*>(smem + L.off_z);
        for (int idx = tid; idx < p.Cz; idx += blockDim.x) z[idx] = __ldg(p.dec_z + idx);
    }
    if (TMA && tid == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kLW);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (TMA && warp == kLW) {
        if (lane == 0) produce<kLTT, true, true>(p, smem + L.off_stage, L.stage_bytes, full, empty, kLW, CB);
        return;
    }

    const int nthr = kLW * 32;
    const int myh = lane / TB, myt = lane % TB;
    int seq = 0;
    bool alive = true;
    WorkCursor wc = work_begin(p);
    ItemRange r;
    while (work_next<true>(p, wc, r)) {
        const int greal = p.G;
        rotate_query<G>(p, r, sR, pitch, sQ, sFin, tid, nthr);
        named_bar_sync(1, nthr);
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
        const int64_t base = (int64_t)r.b * p.kv_bs + (int64_t)r.kvh * p.kv_hs;

        for (int t0 = r.tok0; t0 < r.tok1; t0 += kLTT, ++seq) {
            const int s = seq % p.stages;
            const CT* Kt;
            const CT* Vt;
            if (TMA) {
                if (alive && !mbar_wait(&full[s], (seq / p.stages) & 1, kErrWaitFull)) alive = false;
                Kt = reinterpret_cast<const CT*>(smem + L.off_stage + s * L.stage_bytes);
                Vt = Kt + kLTT * m;
            } else {
                Kt = reinterpret_cast<const CT*>(p.kc) + base + (int64_t)t0 * m;
                Vt = reinterpret_cast<const CT*>(p.vc) + base + (int64_t)t0 * m;
            }
            const int nt = min(kLTT, r.tok1 - t0);
            if (alive) {
                #pragma unroll 1
                for (int blk = 0; blk < 32 / TB; ++blk) {
                    const int tl0 = warp * 32 + blk * TB;
                    if (tl0 >= nt) break;
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
                        if (mn != mrun[g]) {
                            const float alpha = fast_exp2(mrun[g] - mn);
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

        // merge the consumer warps (online-softmax states) into sM / sL / sO
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
        named_bar_sync(1, nthr);
        for (int idx = tid; idx < greal * (dim + 1); idx += nthr) {
            const int g = idx / (dim + 1), k = idx % (dim + 1);
            float M = -INFINITY;
            #pragma unroll
            for (int w = 0; w < kLW; ++w) M = fmaxf(M, sCm[w * G + g]);
            float v = 0.f;
            #pragma unroll
            for (int w = 0; w < kLW; ++w) {
                const float mw = sCm[w * G + g];
                const float f = (mw == -INFINITY) ? 0.f : fast_exp2(mw - M);
                v = fmaf(k == dim ? sCl[w * G + g] : sCo[(w * G + g) * dim + k], f, v);
            }
            if (k == dim) { sL[g] = v; sM[g] = M; } else { sO[g * dim + k] = v; }
        }
        named_bar_sync(1, nthr);
        finish_item(p, r, sM, sL, sO, sFin, sflag, sR, pitch, tid, nthr, 1);
    }
    xr_finish_call(p, sO, sFin, sR, pitch, tid, nthr, 1);
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

// The same merge with each part behind its own pointer: part p of row r at
// part_ptrs[p] + part_offset + r * (dim + 2).  The pointers may name other GPUs'
// memory (peer buffers mapped over NVLink); the loads are plain coherent loads
// that bypass L1 (the buffers are rewritten between calls).
__global__ void __launch_bounds__(128) lse_combine_gather_kernel(const float* const* __restrict__ part_ptrs,
                                                                 int n_parts, int64_t part_offset, int rows,
                                                                 int dim, const float* __restrict__ R,
                                                                 float* __restrict__ out, int64_t out_rs) {
    extern __shared__ float fin_g[];               // [dim]
    const int row = blockIdx.x;
    if (row >= rows) return;
    for (int k = threadIdx.x; k < dim; k += blockDim.x) {
        float M = -INFINITY;
        for (int pi = 0; pi < n_parts; ++pi)
            M = fmaxf(M, __ldcg(part_ptrs[pi] + part_offset + (int64_t)row * (dim + 2)));
        float l = 0.f, v = 0.f;
        for (int pi = 0; pi < n_parts; ++pi) {
            const float* src = part_ptrs[pi] + part_offset + (int64_t)row * (dim + 2);
            const float mp = __ldcg(src);
            const float f = (mp == -INFINITY) ? 0.f : expf(mp - M);
            l = fmaf(__ldcg(src + 1), f, l);
            v = fmaf(__ldcg(src + 2 + k), f, v);
        }
        fin_g[k] = (l > 0.f) ? v / l : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        float v = 0.f;
        for (int k = 0; k < dim; ++k) v = fmaf(fin_g[k], __ldg(R + k * dim + i), v);
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

}  // namespace pkv

#include "pkv_attn_tc.cu"
#include "pkv_attn_mha8.cu"
#include "pkv_attn_mha12.cu"
#include "pkv_attn_gqa12.cu"
#include "pkv_attn_gqa12m.cu"

namespace pkv {

struct AttnPlan {
    bool mha12;                        // attn_mha12_kernel, or with mha12s attn_mha12_stream_kernel
    bool mha12s;
    bool mha8;                         // attn_mha8_kernel
    bool gqa12;                        // attn_gqa12_kernel: four query heads of one KV head per unit
    bool g12m;                         // ... as attn_gqa12_mma_kernel (fp16-pair tensor-core tiles)
    bool polar;                        // attn_polar_kernel, else attn_lut_kernel
    int G, TPL, stages, nsplit, chunk, tt, threads, smem, ctas_per_sm;
    bool tma;
    bool bal;                          // balanced tile ranges instead of round-robin items
    bool qunits;                       // one unit per query head (grouped heads in the one-head kernel)
    bool tc;                           // attn_tc_kernel (tensor cores, bf16/fp16 queries)
    int tpu, seg_cap, slots;           // tiles per unit, tiles per segment at most, partial slots
    int64_t tiles, grid;               // balanced: total tiles, CTAs
};

// Work units per batch row: the KV heads; every query head (grouped heads on the one-head
// kernels); or every four query heads (attn_gqa12_kernel).
static int units_per_row(const AttnPlan& pl, const pkv_attn_args* a) {
    return pl.qunits ? a->q_heads : pl.gqa12 ? a->q_heads / gqa12::HQ : a->kv_heads;
}

static bool tma_ok(const pkv_codec* c, const pkv_attn_args* a) {
    const int row_bytes = (c->dim / 3) * a->code_bytes;
    const uintptr_t kb = reinterpret_cast<uintptr_t>(a->k_codes), vb = reinterpret_cast<uintptr_t>(a->v_codes);
    return (row_bytes % 16 == 0) && (kb % 16 == 0) && (vb % 16 == 0) &&
           ((a->kv_batch_stride * a->code_bytes) % 16 == 0) && ((a->kv_head_stride * a->code_bytes) % 16 == 0);
}

static AttnPlan plan_attn(const pkv_codec* c, const pkv_attn_args* a) {
    AttnPlan pl{};
    const int m = c->dim / 3;
    pl.G = round_group(a->q_heads / a->kv_heads);
    pl.tma = tma_ok(c, a);
    const int Cz = 1 << c->bits_z;
    pl.polar = pl.tma && m <= 32 && c->xy_mode == 0 && c->bits_z <= 4 && (c->bits_r + c->bits_theta) <= 8 &&
               (c->xy_per_z == 0 || c->bias_xy != nullptr);
    pl.mha12 = pl.polar && c->dim == 96 && a->code_bytes == 2 && c->bits_z == 4 && c->bits_r == 4 &&
               c->bits_theta == 4 && c->xy_per_z == 0 && (c->flags & PKV_CODEC_Z_UNIFORM) != 0;
    // grouped heads: every query head streams its KV head's codes on its own (the group's re-reads
    // of the same codes hit L2), which beats per-token work for the whole group at 12-bit codes
    pl.qunits = pl.mha12 && a->q_heads != a->kv_heads;
    // groups of 4, 8, ... query heads: each code decoded once for four heads (measured on B200
    // against one query head per unit, whose decode work grows with the group)
    pl.gqa12 = pl.mha12 && a->q_heads / a->kv_heads >= gqa12::HQ && (a->q_heads / a->kv_heads) % gqa12::HQ == 0;
    if (pl.gqa12) {
        pl.mha12 = false;
        pl.qunits = false;
        // the tensor-core form holds the decoded (x, y) as fp16 pairs: radii up to 2^15
        pl.g12m = (c->flags & PKV_CODEC_FP32_ATTN) == 0 && c->r_max > 0.f && c->r_max <= 32768.f;
    }
    if (pl.mha12) {
        pl.G = 1;
        // measured on B200: the two-pass kernel wins while a unit is one item (phi3-decode,
        // 2.85 vs 2.73 TB/s); past its 4096-token items the one-pass kernel does (longctx
        // 131072 tokens, 1.14 vs 0.87 TB/s)
        pl.mha12s = a->seq_len > mha12::CH;
    }
    {
        const int n_xy = (c->xy_per_z ? Cz : 1) << (c->bits_r + c->bits_theta);
        // measured: grouped heads (one decode per KV token serves the whole group) and per-z-bin
        // tables gain on tensor cores; a single uniform-polar head is faster on the polar kernel
        pl.tc = !pl.mha12 && !pl.gqa12 && pl.tma && c->dim == 96 && (a->q_dtype == PKV_BF16 || a->q_dtype == PKV_F16) &&
                (a->code_bytes == 1 || a->code_bytes == 2) && n_xy <= 4096 && Cz <= 256 &&
                a->q_heads / a->kv_heads <= 16 && (a->q_heads > a->kv_heads || c->xy_per_z != 0);
    }
    // one-byte uniform-polar codes: one query head per unit, unless tensor cores serve the group
    pl.mha8 = pl.polar && !pl.tc && c->dim == 96 && a->code_bytes == 1 && c->xy_per_z == 0 &&
              (c->flags & PKV_CODEC_Z_UNIFORM) != 0 && c->bits_z >= 1 && c->bits_r + c->bits_theta <= 5 &&
              c->bits_z + c->bits_r + c->bits_theta <= 8;
    if (pl.mha8) {
        pl.qunits = a->q_heads != a->kv_heads;
        pl.G = 1;
    }
    if (pl.gqa12) {
        pl.polar = false;
        pl.TPL = 1;
        pl.G = gqa12::HQ;
        pl.tt = pl.g12m ? g12m::TT : gqa12::TT;
        pl.threads = pl.g12m ? g12m::W * 32 + 32 : gqa12::W * 32 + 32;
        pl.stages = pl.g12m ? g12m::SLOTS : gqa12::SLOTS;
        pl.smem = pl.g12m ? g12m::TOTAL : gqa12::TOTAL;
        pl.chunk = 1 << 30;                // online softmax: no cap on the tokens of an item
        pl.ctas_per_sm = 1;
    } else if (pl.tc) {
        pl.polar = false;
        pl.TPL = 1;
        pl.tt = atc::TT;
        {
            const int g = a->q_heads / a->kv_heads;
            pl.G = g <= 4 ? 4 : (g <= 8 ? 8 : 16);          // register state per head of the group
        }
        pl.threads = atc::threads_for(pl.G);
        pl.stages = atc::STAGES;
        pl.smem = atc::SMEM_BYTES;
        pl.chunk = 1 << 30;                // online softmax: no cap on the tokens of an item
        pl.ctas_per_sm = 1;
    } else if (pl.mha8) {
        pl.polar = false;
        pl.TPL = 1;
        pl.tt = mha8::TT;
        pl.threads = mha8::W * 32 + 32;
        pl.stages = mha8::STAGES;
        pl.smem = mha8::TOTAL;
        pl.chunk = 1 << 30;                // online softmax: no cap on the tokens of an item
        pl.ctas_per_sm = 1;
    } else if (pl.mha12s) {
        pl.TPL = 1;
        pl.tt = mha12s::TT;
        pl.threads = mha12s::W * 32 + 32;
        pl.stages = mha12s::STAGES;
        pl.smem = mha12s::TOTAL;
        pl.chunk = 1 << 30;                // online softmax: no cap on the tokens of an item
        pl.ctas_per_sm = 2;
    } else if (pl.mha12) {
        pl.TPL = 1;
        pl.tt = mha12::TT;
        pl.threads = mha12::W * 32 + 32;
        pl.stages = mha12::STAGES;
        pl.smem = mha12::TOTAL;
        pl.chunk = mha12::CH;
        pl.ctas_per_sm = 2;
    } else if (pl.polar) {
        pl.TPL = 1;
        pl.tt = kPTT;
        pl.threads = kPW * 32 + 32;
        pl.stages = (m * a->code_bytes <= 32) ? 4 : 3;
        PolarLayout L = polar_layout(m, a->code_bytes, c->dim, pl.G, c->bits_z, c->bits_r, c->bits_theta, pl.stages);
        pl.smem = L.total;
        pl.chunk = L.chunk;
        pl.ctas_per_sm = 2;
    } else {
        pl.TPL = (m <= 32) ? 1 : 2;
        pl.tt = kLTT;
        pl.threads = pl.tma ? kLW * 32 + 32 : kLW * 32;
        const int n_xy = (c->xy_per_z ? Cz : 1) << (c->bits_r + c->bits_theta);
        pl.stages = (m * a->code_bytes <= 64) ? 4 : 3;
        LutLayout L = lut_layout(m, a->code_bytes, c->dim, pl.G, n_xy, Cz, pl.stages);
        while (L.total > 227 * 1024 && pl.stages > 2) {
            --pl.stages;
            L = lut_layout(m, a->code_bytes, c->dim, pl.G, n_xy, Cz, pl.stages);
        }
        pl.smem = L.total;
        pl.chunk = 1 << 30;
        pl.ctas_per_sm = 2;
    }
    // split count: minimise rounds * (tiles per item + overhead); items carry at most `chunk` tokens
    const int tiles_total = std::max(1, (a->seq_len + pl.tt - 1) / pl.tt);
    const int max_tiles_item = std::max(1, pl.chunk / pl.tt);
    const int64_t units = (int64_t)a->batch * units_per_row(pl, a);
    const int64_t grid = (int64_t)num_sms() * pl.ctas_per_sm;
    // fixed cost of an item in tile units: the tensor-core kernel's items also rotate the group's
    // queries through global R and merge their splits, about eight of its 128-token tiles
    // (query rotation, score table and warp merge: about two tiles of the one-head kernels)
    const double item_cost = pl.tc ? 8.0 : pl.gqa12 ? 3.0 : (pl.mha8 || pl.mha12s) ? 2.0 : 1.0;
    int best = 0;
    double best_cost = 1e300;
    const int min_split = a->num_splits > 0 ? a->num_splits : (tiles_total + max_tiles_item - 1) / max_tiles_item;
    const int max_split = a->num_splits > 0 ? a->num_splits : std::max(min_split, std::min(tiles_total, 64));
    for (int ns = std::max(1, min_split); ns <= max_split; ++ns) {
        const int tiles_per = (tiles_total + ns - 1) / ns;
        if (tiles_per > max_tiles_item) continue;
        const int64_t items = units * ns;
        const int64_t rounds = (items + grid - 1) / grid;
        const double cost = (double)rounds * (tiles_per + item_cost) + (ns > 1 ? 0.25 : 0.0);
        if (cost < best_cost - 1e-9) { best_cost = cost; best = ns; }
    }
    if (best == 0) best = (tiles_total + max_tiles_item - 1) / max_tiles_item;
    pl.chunk = ((tiles_total + best - 1) / best) * pl.tt;
    pl.nsplit = std::max(1, (a->seq_len + pl.chunk - 1) / pl.chunk);
    pl.slots = pl.nsplit;
    pl.bal = false;
    // balanced schedule: every CTA streams the same number of tiles (uniform lengths only); a
    // CTA's range spans at most ceil(per / cap) + 1 segments, each paying the item overhead.
    // Measured on B200: it pays for the one-pass LUT kernel (+12-16 %); the polar and 12-bit
    // kernels' per-item fixed costs (query rotation, score table, score pass) outweigh the
    // balance (phi3-decode: -18 % two-pass, -17 % one-pass).
    if (!pl.polar && !pl.tc && !pl.mha8 && a->seq_lens == nullptr && a->num_splits == 0 && a->seq_len > 0) {
        const int64_t T = units * tiles_total;
        const int64_t G = std::min<int64_t>(grid, T);
        const int64_t per = (T + G - 1) / G;
        const int cap = std::min(max_tiles_item, tiles_total);
        // a CTA's range spans at most ceil(per / cap) + 1 segments; a unit longer than a CTA's
        // share is cut at CTA boundaries only
        const int64_t segs = std::min<int64_t>((per + cap - 1) / cap + 1, per);
        const double cost = (double)per + (double)segs * item_cost + 0.25;
        if (cost < best_cost - 1e-9) {
            pl.bal = true;
            pl.tpu = tiles_total;
            pl.seg_cap = max_tiles_item;
            pl.tiles = T;
            pl.grid = G;
            // cuts inside one unit: chunk ends plus CTA boundaries (at least T / G tiles apart)
            const int64_t spacing = std::max<int64_t>(1, T / G);
            pl.slots = (int)((tiles_total - 1) / max_tiles_item + 1 + (tiles_total - 1) / spacing + 1);
            pl.nsplit = pl.slots;
            pl.chunk = std::min(max_tiles_item, tiles_total) * pl.tt;
        }
    }
    return pl;
}

// Groups above 8 query heads per KV head run only on the kernels that do not unroll over the group.
bool attn_group_supported(const pkv_codec* c, const pkv_attn_args* a) {
    if (a->q_heads / a->kv_heads <= 8) return true;
    const AttnPlan pl = plan_attn(c, a);
    return pl.tc || pl.mha12 || pl.mha8 || pl.gqa12;
}

void describe_attn(const pkv_codec* c, const pkv_attn_args* a, pkv_attn_plan* out) {
    const AttnPlan pl = plan_attn(c, a);
    out->kernel = pl.tc      ? PKV_KERNEL_TC
                  : pl.gqa12 ? (pl.g12m ? PKV_KERNEL_GQA12_MMA : PKV_KERNEL_GQA12)
                  : pl.mha12 ? (pl.mha12s ? PKV_KERNEL_MHA12_STREAM : PKV_KERNEL_MHA12)
                  : pl.mha8  ? PKV_KERNEL_MHA8
                             : (pl.polar ? PKV_KERNEL_POLAR : PKV_KERNEL_LUT);
    out->num_splits = pl.nsplit;
    out->tokens_per_split = pl.chunk;
    out->balanced = pl.bal ? 1 : 0;
    out->threads = pl.threads;
    out->smem_bytes = pl.smem;
    out->ctas_per_sm = pl.ctas_per_sm;
}

// Arrival counters of a split call: one per (batch row, unit head).
size_t attn_counter_bytes(const pkv_codec* c, const pkv_attn_args* a) {
    const AttnPlan pl = plan_attn(c, a);
    return (size_t)a->batch * units_per_row(pl, a) * sizeof(int32_t);
}

size_t attn_workspace_size(const pkv_codec* c, const pkv_attn_args* a) {
    AttnPlan pl = plan_attn(c, a);
    if (!pl.bal && pl.nsplit <= 1) return 0;
    size_t part = (size_t)a->batch * a->q_heads * pl.slots * (c->dim + 2) * sizeof(float);
    part = (part + 255) / 256 * 256;
    return part + (size_t)a->batch * units_per_row(pl, a) * sizeof(int32_t);
}

template <typename K>
static int launch_kernel(K kern, const AttnParams& p, const AttnPlan& pl, cudaStream_t st) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem) != cudaSuccess)
        return PKV_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, pl.threads, pl.smem) != cudaSuccess ||
        per_sm <= 0)
        return PKV_ERR_CUDA;
    int64_t grid = std::min<int64_t>(p.num_items, (int64_t)per_sm * num_sms());
    if (pl.bal) grid = std::min<int64_t>(grid, pl.grid);     // the partition the slots were sized for
    kern<<<(unsigned)grid, pl.threads, pl.smem, st>>>(p);
    return cudaGetLastError() == cudaSuccess ? PKV_OK : PKV_ERR_CUDA;
}

template <int CB, int G>
static int launch_polar_g(const AttnParams& p, const AttnPlan& pl, cudaStream_t st) {
    return p.bias_xy ? launch_kernel(attn_polar_kernel<CB, G, true>, p, pl, st)
                     : launch_kernel(attn_polar_kernel<CB, G, false>, p, pl, st);
}

template <int CB>
static int launch_polar(const AttnParams& p, const AttnPlan& pl, cudaStream_t st) {
    switch (pl.G) {
        case 1: return launch_polar_g<CB, 1>(p, pl, st);
        case 2: return launch_polar_g<CB, 2>(p, pl, st);
        case 4: return launch_polar_g<CB, 4>(p, pl, st);
        case 8: return launch_polar_g<CB, 8>(p, pl, st);
    }
    return PKV_ERR_UNSUPPORTED;
}

template <int CB, int TPL, int G>
static int launch_lut_g(const AttnParams& p, const AttnPlan& pl, cudaStream_t st) {
    return pl.tma ? launch_kernel(attn_lut_kernel<CB, TPL, G, true>, p, pl, st)
                  : launch_kernel(attn_lut_kernel<CB, TPL, G, false>, p, pl, st);
}

template <int CB, int TPL>
static int launch_lut_tpl(const AttnParams& p, const AttnPlan& pl, cudaStream_t st) {
    switch (pl.G) {
        case 1: return launch_lut_g<CB, TPL, 1>(p, pl, st);
        case 2: return launch_lut_g<CB, TPL, 2>(p, pl, st);
        case 4: return launch_lut_g<CB, TPL, 4>(p, pl, st);
        case 8: return launch_lut_g<CB, TPL, 8>(p, pl, st);
    }
    return PKV_ERR_UNSUPPORTED;
}

template <int CB>
static int launch_lut(const AttnParams& p, const AttnPlan& pl, cudaStream_t st) {
    return pl.TPL == 1 ? launch_lut_tpl<CB, 1>(p, pl, st) : launch_lut_tpl<CB, 2>(p, pl, st);
}

// Split-sequence exchange buffer of one rank: partial slots [world][rows][dim + 2], output rows
// [rows][dim], one arrival counter per unit, then the done and CTA counters; 256-byte aligned parts.
// Exchange buffer of a rank: partial slots [2 parities][world][rows][dim + 2] of flagged 8-byte
// words, output rows [rows][dim] f32, control words (epoch, CTA count).
struct XrLayout { size_t out_off, ctl_off, bytes; int rows, units; };

static XrLayout xr_layout_of(const pkv_codec* c, const pkv_attn_args* a, const AttnPlan& pl, int world) {
    auto up = [](size_t x) { return (x + 255) / 256 * 256; };
    XrLayout L{};
    L.rows = a->batch * a->q_heads;
    L.units = a->batch * units_per_row(pl, a);
    L.out_off = up((size_t)2 * world * L.rows * (c->dim + 2) * sizeof(uint64_t));
    L.ctl_off = L.out_off + up((size_t)L.rows * c->dim * sizeof(float));
    L.bytes = L.ctl_off + 256;
    return L;
}

void xr_layout(const pkv_codec* c, const pkv_attn_args* a, int world, pkv_xr_layout* out) {
    const XrLayout L = xr_layout_of(c, a, plan_attn(c, a), world);
    out->bytes = L.bytes;
    out->out_offset = L.out_off;
    out->rows = L.rows;
    out->units = L.units;
}

// Byte offset and length of what pkv_xr_reset zeroes: the whole buffer (slots, whose stale flags
// must not match the restarted epochs, outputs and control words).
void xr_counter_span(const pkv_codec* c, const pkv_attn_args* a, int world, size_t* off, size_t* len) {
    const XrLayout L = xr_layout_of(c, a, plan_attn(c, a), world);
    *off = 0;
    *len = L.bytes;
}

int launch_attn(const pkv_codec* c, const pkv_attn_args* a, void* ws, size_t ws_bytes, cudaStream_t st,
                const pkv_exchange* xr) {
    AttnPlan pl = plan_attn(c, a);
    if (a->q_heads / a->kv_heads > 8 && !pl.tc && !pl.mha12 && !pl.mha8 && !pl.gqa12) return PKV_ERR_UNSUPPORTED;
    if (pl.smem > 227 * 1024) return PKV_ERR_UNSUPPORTED;
    AttnParams p{};
    p.B = a->batch; p.Hq = a->q_heads; p.Hkv = a->kv_heads; p.S = a->seq_len;
    p.G = pl.qunits ? 1 : pl.gqa12 ? gqa12::HQ : a->q_heads / a->kv_heads; p.m = c->dim / 3; p.dim = c->dim;
    p.Hu = units_per_row(pl, a);
    p.Gq = pl.qunits ? a->q_heads / a->kv_heads : pl.gqa12 ? a->q_heads / a->kv_heads / gqa12::HQ : 1;
    p.q = a->q; p.qdt = a->q_dtype; p.q_bs = a->q_batch_stride; p.q_hs = a->q_head_stride;
    p.kc = static_cast<const uint8_t*>(a->k_codes); p.vc = static_cast<const uint8_t*>(a->v_codes);
    p.kv_bs = a->kv_batch_stride; p.kv_hs = a->kv_head_stride;
    p.seq_lens = a->seq_lens;
    p.scale_log2 = a->scale * kLog2e;
    p.out = a->out; p.out_bs = a->out_batch_stride; p.out_hs = a->out_head_stride;
    p.nsplit = pl.nsplit; p.chunk = pl.chunk;
    p.partial_only = a->partial_only; p.partial_out = a->partial_out;
    p.bal = pl.bal ? 1 : 0;
    p.slots = pl.slots;
    p.tt = pl.tt; p.tpu = pl.tpu; p.seg_cap = pl.seg_cap; p.tiles = pl.bal ? pl.tiles : 0;
    if (pl.bal || pl.nsplit > 1) {
        size_t need = attn_workspace_size(c, a);
        if (!ws || ws_bytes < need) return PKV_ERR_WORKSPACE;
        size_t part = (size_t)a->batch * a->q_heads * pl.slots * (c->dim + 2) * sizeof(float);
        part = (part + 255) / 256 * 256;
        p.ws_part = static_cast<float*>(ws);
        p.ws_count = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ws) + part);
    }
    p.R = c->R; p.dec_z = c->dec_z; p.dec_xy = c->dec_xy; p.bias_xy = c->bias_xy;
    p.bits_z = c->bits_z; p.bits_r = c->bits_r; p.bits_t = c->bits_theta;
    p.bits_flat = c->bits_r + c->bits_theta;
    p.code_mask = (1 << (c->bits_z + p.bits_flat)) - 1;
    p.flat_mask = (1 << p.bits_flat) - 1;
    p.xy_per_z = c->xy_per_z;
    p.Cz = 1 << c->bits_z;
    p.n_xy = (c->xy_per_z ? p.Cz : 1) << p.bits_flat;
    p.r_max = c->r_max;
    p.num_items = pl.bal ? (int)std::min<int64_t>(pl.tiles, INT32_MAX) : a->batch * p.Hu * pl.nsplit;
    p.stages = pl.stages;
    if (xr) {
        const XrLayout L = xr_layout_of(c, a, pl, xr->world);
        p.xr_world = xr->world;
        p.xr_rank = xr->rank;
        p.xr_units = L.units;
        for (int s = 0; s < xr->world; ++s) p.xr_buf[s] = static_cast<uint8_t*>(xr->buffers[s]);
        p.xr_out_off = (int64_t)L.out_off;
        p.xr_ctl_off = (int64_t)L.ctl_off;
        p.xr_wait_ns = (uint64_t)xr->wait_limit_us * 1000ull;
        p.partial_only = 0;
        p.out = nullptr;
        if (p.num_items == 0) {
            // an empty shard still publishes an empty partial (m = -inf, l = 0) for every unit
            // and merges its outputs: one empty item per unit
            p.bal = 0;
            p.nsplit = 1;
            p.chunk = 1;
            p.num_items = a->batch * p.Hu;
        }
    }
    if (p.num_items == 0) return PKV_OK;
    if (pl.tc) {
        if (a->code_bytes == 1)
            return pl.G == 4 ? launch_kernel(attn_tc_kernel<1, 4>, p, pl, st)
                             : pl.G == 8 ? launch_kernel(attn_tc_kernel<1, 8>, p, pl, st)
                                         : launch_kernel(attn_tc_kernel<1, 16>, p, pl, st);
        return pl.G == 4 ? launch_kernel(attn_tc_kernel<2, 4>, p, pl, st)
                         : pl.G == 8 ? launch_kernel(attn_tc_kernel<2, 8>, p, pl, st)
                                     : launch_kernel(attn_tc_kernel<2, 16>, p, pl, st);
    }
    if (pl.gqa12) return pl.g12m ? launch_kernel(attn_gqa12_mma_kernel, p, pl, st)
                                 : launch_kernel(attn_gqa12_kernel, p, pl, st);
    if (pl.mha12s) return launch_kernel(attn_mha12_stream_kernel, p, pl, st);
    if (pl.mha12) return launch_kernel(attn_mha12_kernel, p, pl, st);
    if (pl.mha8) return launch_kernel(attn_mha8_kernel, p, pl, st);
    if (pl.polar) return a->code_bytes == 1 ? launch_polar<1>(p, pl, st) : launch_polar<2>(p, pl, st);
    return a->code_bytes == 1 ? launch_lut<1>(p, pl, st) : launch_lut<2>(p, pl, st);
}

int launch_lse_combine(const pkv_codec* c, const float* parts, int n_parts, int64_t part_stride,
                       int rows, float* out, int64_t out_rs, cudaStream_t st) {
    if (rows == 0) return PKV_OK;
    lse_combine_kernel<<<rows, 128, c->dim * sizeof(float), st>>>(parts, n_parts, part_stride, rows, c->dim,
                                                                   c->R, out, out_rs);
    return cudaGetLastError() == cudaSuccess ? PKV_OK : PKV_ERR_CUDA;
}

int launch_lse_combine_gather(const pkv_codec* c, const float* const* part_ptrs, int n_parts, int64_t part_offset,
                              int rows, float* out, int64_t out_rs, cudaStream_t st) {
    if (rows == 0) return PKV_OK;
    lse_combine_gather_kernel<<<rows, 128, c->dim * sizeof(float), st>>>(part_ptrs, n_parts, part_offset, rows,
                                                                          c->dim, c->R, out, out_rs);
    return cudaGetLastError() == cudaSuccess ? PKV_OK : PKV_ERR_CUDA;
}

}  // namespace pkv
