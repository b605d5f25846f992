// pkv_attn_gqa12m.cu -- decode attention for grouped query heads over 12-bit (4+4+4) uniform-polar
// codes of head_dim 96, with both contractions (q . k over the 96 dims, p . v over the tokens) on
// the tensor cores as register-operand mma.sync tiles.  One work unit is four query heads of one
// KV head (as in attn_gqa12_kernel); each code is decoded once, straight into an operand fragment.
//
// Why register-operand tiles and not tcgen05: a unit's four heads are the narrow side of both
// products (n = 8 columns here; tcgen05 wants M >= 64 and operands in shared or tensor memory),
// and the operands are produced by a table decode in registers.  Staging the decoded tiles
// through shared memory for tcgen05 costs more issue slots and shared bandwidth than the
// products themselves (the attn_tc_kernel design), so here the decode feeds the tiles directly.
//
// Numerics: every operand is an fp16 pair (hi, lo) with hi + lo equal to the fp32 value to about
// 2^-22, and the pair rides either along the contraction or across the eight output columns:
//  * the decoded (x, y) of a code sit in a table as (x_hi, x_lo), (y_hi, y_lo); a fragment's
//    k-pair (2c, 2c + 1) is one such pair, so the product sums x_hi b + x_lo b;
//  * the queries (and the softmax weights) enter as eight columns: column h < 4 holds head h's hi
//    part and column h + 4 its lo part; the two columns are added once (scores per tile, output
//    rows per item).  All four cross products are thus kept; products and sums are fp32.
//  * z enters through its integer bin index i_z (exact): uniform bins are affine in i_z (z = z0 +
//    dz i_z), so q . z = z0 sum q_z + dz sum q_z i_z, with i_z as the fp16 subnormal i_z 2^-24 of
//    one byte permute, and o_z = (z0 + 8 dz) l + dz sum p (i_z - 8), with i_z - 8 as an exact fp16.
//    The centring matters: the tensor-core sums truncate, and an uncentred sum p i_z grows with
//    every token while the result is a small difference of it and z0 l.
//  * the queries are scaled by a power of two per item (their largest |value| lands in
//    [2^13, 2^14)) and the scores scaled back in the exponent; the weights are 2^12 exp2(s - m),
//    which keeps them normal in fp16 down to 2^-26 of the largest.
// The result is within a few 1e-6 of the fp64 softmax(q . decode(K)^T * scale) . decode(V)
// (polar_attention.py:277-309 with decoded values) for head_dim 96 data.
//
// Layout of a warp's 16 tokens of a tile (lane = 4 g + c):
//  * scores: rows = tokens, k = dims.  Lane (g, c) decodes tokens rho(g), rho(g) + 8 with
//    rho(g) = (g >> 1) + 4 (g & 1), triplets 8c .. 8c + 7 (one 16-byte load a token): k-step j
//    < 8 is the (x, y) pair of triplet 8c + j, k-steps 8, 9 the z indices of triplets 8c + 4j'
//    .. 8c + 4j' + 3.  The permutation of the dims is the same for the query fragments.
//  * weights: the score tile (rows = tokens rho(.), columns = head parts) is turned into the
//    p . v operand by two 8x8 transposes (movmatrix): lane (g, c) then holds column g of tokens
//    (c, c + 4) and (c + 8, c + 12).
//  * values: rows = dims, k = tokens.  For (x, y) the k-pairs are (token, hi/lo), so a step
//    covers 8 tokens and the weight operand is (p, p); rows g / g + 8 are x / y of triplet 4g + m
//    (m-tile m < 4).  For z the k-pairs are two tokens and rows g / g + 8 are the z of triplets
//    4g + 2m', 4g + 2m' + 1 (m-tiles 4, 5).  Lane (g, c) reads tokens c, c + 4, c + 8, c + 12,
//    triplets 4g .. 4g + 3 (one 8-byte load a token).
// Table lookups: 256 rows (the flat index (i_r << 4) | i_theta) of 32 copies, copy l at bytes
// 8 l of the row, so a warp's 32 loads always take the minimum two wavefronts; the table sits at
// a 64 KB-aligned shared address, so one byte permute of the code word and a per-lane register
// gives the whole address.
//
// Work, ring and exchange as in attn_gqa12_kernel: one CTA per SM (15 consumer warps, one TMA
// producer warp: four warps per SM sub-partition leave 128 registers a thread), persistent over
// balanced tile ranges.  A warp owns two 16-token groups of every tile, interleaved, so that
// each group's tiles hide the other's latencies and the ring bookkeeping is paid per 32 tokens.
// Half tiles (K or V codes of 480 tokens, 30 KB) flow through a ring of four slots (two below the
// table, two above), bounded mbarrier waits; splits merge in the last CTA (finish_item).  R is
// read through L2 (the query rotation and the final o @ R), which leaves the room to the ring.

namespace pkv {
namespace g12m {
constexpr int W = 15;                                   // consumer warps (16 warps: 128 registers)
constexpr int HQ = 4;                                   // query heads per unit
constexpr int NG = 2;                                   // 16-token groups per warp per tile
constexpr int TW = 16 * NG;                             // tokens per warp per tile
constexpr int TT = W * TW;                              // tokens per tile
constexpr int HALF = TT * 64;                           // K (or V) codes of a tile: 32 x uint16 / token
constexpr int SLOTS = 4;                                // ring of half tiles
constexpr int PF = 1;                                   // tiles asked into L2 ahead of the ring
constexpr int TAB_BYTES = 256 * 32 * 8;                 // [256 flat][32 copies] (x hi|lo, y hi|lo)
// The dynamic shared window of a kernel without static shared memory starts at shared address
// 0x400 on sm_100 (the first KB is reserved; checked at run time).  The table must start at a
// 64 KB-aligned shared address, so it sits at window offset 0x10000 - 0x400; two ring slots and
// the queries fill the window below it, the rest (two more slots among it) lies above.
constexpr uint32_t SMEM_BASE = 0x400;
constexpr int OFF_TAB = (int)((0x10000u - (SMEM_BASE & 0xFFFFu)) & 0xFFFFu);
constexpr int SLOTS_LO = 2;                             // ring slots below the table
constexpr int OFF_RING_LO = 0;
constexpr int OFF_Q = OFF_RING_LO + SLOTS_LO * HALF;    // [4][96] rotated, scaled queries
constexpr int OFF_QRAW = OFF_Q + HQ * 96 * 4;           // [4][96] raw queries
constexpr int OFF_ACC = OFF_TAB + TAB_BYTES;            // item merge [W][4][96]
constexpr int OFF_WML = OFF_ACC + W * HQ * 96 * 4;      // [W][4] max, [W][4] sum
constexpr int OFF_FIN = OFF_WML + 2 * W * HQ * 4;       // [4][96]
constexpr int OFF_MISC = OFF_FIN + HQ * 96 * 4;         // sM[4], sL[4], sC[4], flag, amax[W]
constexpr int OFF_BAR = OFF_MISC + 128;                 // full[SLOTS], empty[SLOTS]
constexpr int OFF_RING_HI = (OFF_BAR + 2 * SLOTS * 8 + 127) / 128 * 128;
constexpr int TOTAL = OFF_RING_HI + (SLOTS - SLOTS_LO) * HALF;
static_assert(OFF_QRAW + HQ * 96 * 4 <= OFF_TAB, "slots and queries below the table");
static_assert(OFF_ACC % 16 == 0 && OFF_BAR % 8 == 0 && HALF % 128 == 0, "alignment");
static_assert(TOTAL <= 227 * 1024, "one CTA per SM");
static_assert(W * 32 >= HQ * 96, "one consumer thread per query element (the query prefetch)");
static_assert((W + 1) * 32 == 2 * 256, "two threads per table row in the fill");

// window offset of ring slot s
__host__ __device__ constexpr int ring_off(int s) {
    return s < SLOTS_LO ? OFF_RING_LO + s * HALF : OFF_RING_HI + (s - SLOTS_LO) * HALF;
}
}  // namespace g12m

// (hi, lo) fp16 pair of an fp32 value: hi in the low half (k-pair element 2c), lo in the high half
__device__ __forceinline__ uint32_t h2_split(float v) {
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(v - __half2float(hi));
    return (uint32_t)__half_as_ushort(hi) | ((uint32_t)__half_as_ushort(lo) << 16);
}

// the hi (or lo) fp16 part of v, in both halves
__device__ __forceinline__ uint32_t h2_dup_part(float v, bool lo) {
    const __half hi = __float2half_rn(v);
    const __half pt = lo ? __float2half_rn(v - __half2float(hi)) : hi;
    const uint32_t u = __half_as_ushort(pt);
    return u | (u << 16);
}

// the hi (or lo) parts of a and b as one pair (a low, b high)
__device__ __forceinline__ uint32_t h2_pair_part(float a, float b, bool lo) {
    const __half ah = __float2half_rn(a), bh = __float2half_rn(b);
    const __half ap = lo ? __float2half_rn(a - __half2float(ah)) : ah;
    const __half bp = lo ? __float2half_rn(b - __half2float(bh)) : bh;
    return (uint32_t)__half_as_ushort(ap) | ((uint32_t)__half_as_ushort(bp) << 16);
}

// d += a . b on one m16n8k16 tile, fp16 operands, fp32 accumulators
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

__device__ __forceinline__ uint4 lds_u32x4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint2 lds_u32x2m(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

// byte permute with the PTX selector semantics (a selector nibble with bit 3 set replicates the
// sign bit of the selected byte)
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// (i_a - 8, i_b - 8) as fp16 from the low nibbles of bytes 0 and 2 (the i_z of two codes)
__device__ __forceinline__ uint32_t zc8(uint32_t t) {
    const uint32_t h = (t & 0x000F000Fu) | 0x64006400u;      // 1024 + i, exact
    const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h), __halves2half2(__ushort_as_half(0x6408u),
                                                                                  __ushort_as_half(0x6408u)));
    return *reinterpret_cast<const uint32_t*>(&r);
}

__device__ __forceinline__ uint32_t f2h2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// Producer: half tiles in consumption order (K of tile t, then V of tile t) into the ring.  The
// ring holds three tiles; the codes of the next PF tiles of the item are asked into L2 ahead
// (bulk prefetches, no shared memory), so that the copies into the ring meet L2 latency and the
// memory system sees the ring's bytes plus PF tiles in flight per SM.
__device__ void produce_g12m(const AttnParams& p, uint8_t* smem, uint64_t* full, uint64_t* empty) {
    using namespace g12m;
    int seq = 0, s = 0;
    uint32_t phase = 0;                                   // phase of slot s's next fill
    bool ok = true;
    WorkCursor wc = work_begin(p);
    ItemRange r;
    while (ok && work_next<true>(p, wc, r)) {
        const int64_t base = ((int64_t)r.b * p.kv_bs + (int64_t)r.kvh * p.kv_hs) * 2;
        if (PF > 0 && r.tok1 > r.tok0) {                  // (ragged rows leave items empty or inverted)
            const uint32_t bytes = (uint32_t)min(PF * TT, r.tok1 - r.tok0) * 64u;
            bulk_prefetch_l2(p.kc + base + (int64_t)r.tok0 * 64, bytes);
            bulk_prefetch_l2(p.vc + base + (int64_t)r.tok0 * 64, bytes);
        }
        for (int t0 = r.tok0; t0 < r.tok1 && ok; t0 += TT) {
            const uint32_t bytes = (uint32_t)min(TT, r.tok1 - t0) * 64u;
            const int64_t off = base + (int64_t)t0 * 64;
            if (PF > 0 && t0 + PF * TT < r.tok1) {
                const int tp = t0 + PF * TT;
                const uint32_t pbytes = (uint32_t)min(TT, r.tok1 - tp) * 64u;
                bulk_prefetch_l2(p.kc + base + (int64_t)tp * 64, pbytes);
                bulk_prefetch_l2(p.vc + base + (int64_t)tp * 64, pbytes);
            }
            #pragma unroll 1
            for (int h = 0; h < 2; ++h) {
                if (seq >= SLOTS && !mbar_wait(&empty[s], phase ^ 1u, kErrWaitEmpty)) { ok = false; break; }
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s(smem + ring_off(s), (h ? p.vc : p.kc) + off, bytes, &full[s]);
                ++seq;
                if (++s == SLOTS) { s = 0; phase ^= 1u; }
            }
        }
    }
    const int issued = seq;                               // drain before the CTA may exit
    for (int q = max(0, issued - SLOTS); q < issued; ++q)
        mbar_wait(&full[q % SLOTS], (q / SLOTS) & 1, kErrWaitDrain);
}

__global__ void __launch_bounds__(g12m::W * 32 + 32, 1) attn_gqa12_mma_kernel(AttnParams p) {
    using namespace g12m;
    extern __shared__ __align__(128) uint8_t g12m_smem[];
    uint8_t* smem = g12m_smem;
    float* sQ = reinterpret_cast<float*>(smem + OFF_Q);
    float* sQraw = reinterpret_cast<float*>(smem + OFF_QRAW);
    float* sWm = reinterpret_cast<float*>(smem + OFF_WML);
    float* sWl = sWm + W * HQ;
    float* sFin = reinterpret_cast<float*>(smem + OFF_FIN);
    float* sAcc = reinterpret_cast<float*>(smem + OFF_ACC);
    float* sM = reinterpret_cast<float*>(smem + OFF_MISC);
    float* sL = sM + 4;
    float* sC = sM + 8;
    int* sflag = reinterpret_cast<int*>(sM + 12);
    float* sAmax = sM + 16;                               // [W]
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* empty = full + SLOTS;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t smem_base = (uint32_t)__cvta_generic_to_shared(smem);
    const uint32_t tab_addr = smem_base + OFF_TAB;
    if ((tab_addr & 0xFFFFu) != 0u) {                     // the window moved: refuse, loudly
        if (tid == 0) flag_error(kErrSmemLayout);
        return;
    }
    const float z0 = __ldg(p.dec_z), dz = __ldg(p.dec_z + 1) - z0;      // uniform z bins: z = z0 + i dz

    if (tid == 0) {
        for (int s = 0; s < SLOTS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        fence_mbar_init();
    }
    // A partial tile's tail in the ring holds stale or never-written bytes; every decode of a code
    // byte is finite whatever it holds (table rows, masked z nibbles, z bytes as small fp16
    // subnormals), and tokens past the end get score -inf and weight 0, so the ring needs no
    // clearing.
    //
    // The CTA's first global loads in flight at once: the first item's queries, the decode grid
    // for the table, and R asked into L2 for the first query rotation.
    float qreg = 0.f;
    {
        WorkCursor pc = work_begin(p);
        ItemRange r0;
        if (tid < HQ * 96 && work_next<true>(p, pc, r0))
            qreg = q_load(p.q, p.qdt, (int64_t)r0.b * p.q_bs + (int64_t)(r0.hk * HQ + tid / 96) * p.q_hs + tid % 96);
    }
    if (tid < 96 * 96 * 4 / 128) prefetch_l2(reinterpret_cast<const uint8_t*>(p.R) + tid * 128);
    // (x, y) table: row e = (i_r << 4) | i_theta, 32 copies of ((x_hi, x_lo), (y_hi, y_lo)) of the
    // codec's decoded (x, y) of the flat index (the uniform polar grid, stacked_plane.py:297-310)
    // (two threads a row, one load each: the fill costs one L2 round trip)
    {
        const int e = tid >> 1, half = tid & 1;
        const float2 xy = __ldg(reinterpret_cast<const float2*>(p.dec_xy) + e);
        const uint2 v = make_uint2(h2_split(xy.x), h2_split(xy.y));
        uint4* row = reinterpret_cast<uint4*>(smem + OFF_TAB + e * 256 + half * 128);
        #pragma unroll
        for (int k = 0; k < 8; ++k) row[k] = make_uint4(v.x, v.y, v.x, v.y);
    }
    __syncthreads();
    if (warp == W) {
        if (lane == 0) produce_g12m(p, smem, full, empty);
        return;
    }

    constexpr int nthr = W * 32;
    const int g = lane >> 2, c = lane & 3, hp = c & 1;
    const bool lo_col = g >= 4;                           // this lane's operand column is a lo part
    const int qh = g & 3;                                 // ... of head qh
    const int rho = (g >> 1) + 4 * (g & 1);               // score rows g, g + 8: tokens rho, rho + 8
    const uint32_t lanereg = tab_addr | ((uint32_t)lane << 3);
    const uint32_t k_lane = (uint32_t)(rho * 64 + c * 16);
    const uint32_t v_lane = (uint32_t)(c * 64 + g * 8);
    int slot = 0;                                         // ring slot of the next half tile, its fill phase
    uint32_t phase = 0;
    bool alive = true;
    WorkCursor wc = work_begin(p);
    ItemRange r;
    while (work_next<true>(p, wc, r)) {
        const int ntok = r.tok1 - r.tok0;
        const int ntiles = (ntok + TT - 1) / TT;
        // q'_h = scale log2(e) R q_h: one warp per row k of R (read through L2, all of the warp's
        // rows in flight at once, issued before the barrier that publishes the raw queries),
        // lanes over the input index; the four heads' sums finish in a transpose-reduce, then a
        // butterfly over the low three lane bits
        constexpr int RPW = (96 + W - 1) / W;              // rows of R per warp
        float rr[RPW][3];
        #pragma unroll
        for (int i = 0; i < RPW; ++i) {
            const int k = min(warp + i * W, 95);
            #pragma unroll
            for (int u = 0; u < 3; ++u) rr[i][u] = __ldg(p.R + k * 96 + lane + 32 * u);
        }
        if (tid < HQ * 96) sQraw[tid] = qreg;
        named_bar_sync(1, nthr);
        #pragma unroll
        for (int i = 0; i < RPW; ++i) {
            const int k = warp + i * W;
            if (k >= 96) break;
            const float r0 = rr[i][0], r1 = rr[i][1], r2 = rr[i][2];
            float a[HQ];
            #pragma unroll
            for (int h = 0; h < HQ; ++h)
                a[h] = fmaf(r0, sQraw[h * 96 + lane], fmaf(r1, sQraw[h * 96 + lane + 32], r2 * sQraw[h * 96 + lane + 64]));
            const bool up16 = (lane & 16) != 0;
            const float k0 = up16 ? a[2] : a[0], k1 = up16 ? a[3] : a[1];
            const float s0 = up16 ? a[0] : a[2], s1 = up16 ? a[1] : a[3];
            float b0 = k0 + __shfl_xor_sync(0xffffffffu, s0, 16);
            float b1 = k1 + __shfl_xor_sync(0xffffffffu, s1, 16);
            const bool up8 = (lane & 8) != 0;
            float v = (up8 ? b1 : b0) + __shfl_xor_sync(0xffffffffu, up8 ? b0 : b1, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            if ((lane & 7) == 0) sQ[((lane >> 3) & 3) * 96 + k] = v * p.scale_log2;
        }
        named_bar_sync(1, nthr);
        // largest operand magnitude: |q'_x|, |q'_y| and |q'_z| dz
        {
            float a = 0.f;
            if (tid < HQ * 96) a = fabsf(sQ[tid]) * ((tid % 3 == 0) ? fabsf(dz) : 1.f);
            #pragma unroll
            for (int off = 16; off >= 1; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
            if (lane == 0) sAmax[warp] = a;
        }
        // C_h = z0 sum_j q'_h,z,j (true log2 units)
        if (warp < HQ) {
            float cz = sQ[warp * 96 + 3 * lane];
            #pragma unroll
            for (int off = 16; off >= 1; off >>= 1) cz += __shfl_xor_sync(0xffffffffu, cz, off);
            if (lane == 0) sC[warp] = cz * z0;
        }
        named_bar_sync(1, nthr);
        // power-of-two operand scale su = 2^k putting the largest magnitude in [2^13, 2^14)
        float su = 1.f, us = 1.f;
        {
            float amax = 0.f;
            #pragma unroll
            for (int w = 0; w < W; ++w) amax = fmaxf(amax, sAmax[w]);
            if (amax > 0.f && amax <= 3.0e38f) {
                const int e = (int)((__float_as_uint(amax) >> 23) & 0xFF) - 127;   // floor(log2 amax), normal amax
                const int k = max(-120, min(120, 13 - max(e, -126)));
                su = __uint_as_float((uint32_t)(127 + k) << 23);
                us = __uint_as_float((uint32_t)(127 - k) << 23);
            }
        }
        // score operand fragments of this lane: column g (head qh, part lo_col), k-pairs as above
        uint32_t bq[8][2], bz[2][2];
        #pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int t = 8 * c + j;
            bq[j][0] = h2_dup_part(sQ[qh * 96 + 3 * t + 1] * su, lo_col);
            bq[j][1] = h2_dup_part(sQ[qh * 96 + 3 * t + 2] * su, lo_col);
        }
        #pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int t = 8 * c + 4 * j;
            const float sz = su * dz;
            bz[j][0] = h2_pair_part(sQ[qh * 96 + 3 * t] * sz, sQ[qh * 96 + 3 * (t + 1)] * sz, lo_col);
            bz[j][1] = h2_pair_part(sQ[qh * 96 + 3 * (t + 2)] * sz, sQ[qh * 96 + 3 * (t + 3)] * sz, lo_col);
        }
        // softmax state of this lane's heads 2 hp, 2 hp + 1 (true log2 units)
        const float cz0 = sC[2 * hp], cz1 = sC[2 * hp + 1];
        float M0 = -INFINITY, M1 = -INFINITY;
        float thr0 = -INFINITY, thr1 = -INFINITY;         // score-tile value above which M grows
        f32x2 negoff = f2_pack(-INFINITY, -INFINITY);     // cz + 12 - M, or -inf while M is
        const f32x2 uu = f2_pack(us, us);
        f32x2 lsum = f2_pack(0.f, 0.f);
        float acc[6][4];
        #pragma unroll
        for (int m = 0; m < 6; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;

        for (int tile = 0; tile < ntiles; ++tile) {
            const int nt = min(TT, ntok - tile * TT);
            const int wt0 = warp * TW;                      // this warp's first token of the tile
            // ---- scores of 2 x 16 tokens x 8 columns ----------------------------------------
            int s = slot;
            if (alive && !mbar_wait(&full[s], phase, kErrWaitFull)) alive = false;
            alive = __all_sync(0xffffffffu, alive);       // the tiles below are warp-collective
            const bool act = alive && wt0 < nt;
            float T[NG][4];
            #pragma unroll
            for (int gi = 0; gi < NG; ++gi) T[gi][0] = T[gi][1] = T[gi][2] = T[gi][3] = -INFINITY;
            if (act) {
                const uint32_t kb = smem_base + ring_off(s) + wt0 * 64 + k_lane;
                uint32_t kw[NG][2][4];                      // [group][token rho / rho + 8][word]
                #pragma unroll
                for (int gi = 0; gi < NG; ++gi) {
                    const uint4 w0 = lds_u32x4(kb + gi * 1024), w1 = lds_u32x4(kb + gi * 1024 + 512);
                    kw[gi][0][0] = w0.x; kw[gi][0][1] = w0.y; kw[gi][0][2] = w0.z; kw[gi][0][3] = w0.w;
                    kw[gi][1][0] = w1.x; kw[gi][1][1] = w1.y; kw[gi][1][2] = w1.z; kw[gi][1][3] = w1.w;
                }
                // per group two independent chains over the (x, y) steps (even / odd triplets), one for z
                float sxa[NG][4], sxb[NG][4], sz[NG][4];
                #pragma unroll
                for (int gi = 0; gi < NG; ++gi)
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) sxa[gi][i] = sxb[gi][i] = sz[gi][i] = 0.f;
                #pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t sel = (j & 1) ? 0x7624u : 0x7604u;
                    #pragma unroll
                    for (int gi = 0; gi < NG; ++gi) {
                        const uint2 e0 = lds_u32x2m(__byte_perm(kw[gi][0][j >> 1], lanereg, sel));
                        const uint2 e1 = lds_u32x2m(__byte_perm(kw[gi][1][j >> 1], lanereg, sel));
                        mma16816((j & 1) ? sxb[gi] : sxa[gi], e0.x, e1.x, e0.y, e1.y, bq[j][0], bq[j][1]);
                    }
                }
                #pragma unroll
                for (int j = 0; j < 2; ++j)
                    #pragma unroll
                    for (int gi = 0; gi < NG; ++gi) {
                        // (i_z of the low code, i_z of the high code) as fp16 subnormals i_z 2^-24
                        // (bytes 1 and 3 of the word, zero bytes from the second operand)
                        mma16816(sz[gi], prmt(kw[gi][0][2 * j], 0u, 0x4341u), prmt(kw[gi][1][2 * j], 0u, 0x4341u),
                                 prmt(kw[gi][0][2 * j + 1], 0u, 0x4341u), prmt(kw[gi][1][2 * j + 1], 0u, 0x4341u),
                                 bz[j][0], bz[j][1]);
                    }
                #pragma unroll
                for (int gi = 0; gi < NG; ++gi) {
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) T[gi][i] = fmaf(sz[gi][i], 16777216.f, sxa[gi][i] + sxb[gi][i]);
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) T[gi][i] += __shfl_xor_sync(0xffffffffu, T[gi][i], 2);   // hi + lo
                    const int t0 = wt0 + 16 * gi + rho;
                    if (t0 >= nt) T[gi][0] = T[gi][1] = -INFINITY;
                    if (t0 + 8 >= nt) T[gi][2] = T[gi][3] = -INFINITY;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++slot == SLOTS) { slot = 0; phase ^= 1u; }
            // ---- online softmax per head ------------------------------------------------
            uint32_t pA[NG], pB[NG];                        // weight fragments after the transposes
            #pragma unroll
            for (int gi = 0; gi < NG; ++gi) pA[gi] = pB[gi] = 0u;
            if (act) {
                bool up = false;
                #pragma unroll
                for (int gi = 0; gi < NG; ++gi)
                    up = up || T[gi][0] > thr0 || T[gi][2] > thr0 || T[gi][1] > thr1 || T[gi][3] > thr1;
                if (__any_sync(0xffffffffu, up)) {
                    float mx0 = fmaxf(T[0][0], T[0][2]), mx1 = fmaxf(T[0][1], T[0][3]);
                    #pragma unroll
                    for (int gi = 1; gi < NG; ++gi) {
                        mx0 = fmaxf(mx0, fmaxf(T[gi][0], T[gi][2]));
                        mx1 = fmaxf(mx1, fmaxf(T[gi][1], T[gi][3]));
                    }
                    #pragma unroll
                    for (int off = 4; off <= 16; off <<= 1) {
                        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
                    }
                    const float n0 = fmaxf(M0, fmaf(mx0, us, cz0)), n1 = fmaxf(M1, fmaf(mx1, us, cz1));
                    const float f0 = (M0 == -INFINITY) ? 0.f : fast_exp2(M0 - n0);
                    const float f1 = (M1 == -INFINITY) ? 0.f : fast_exp2(M1 - n1);
                    lsum = f2_mul(lsum, f2_pack(f0, f1));
                    #pragma unroll
                    for (int m = 0; m < 6; ++m) {
                        acc[m][0] *= f0; acc[m][1] *= f1; acc[m][2] *= f0; acc[m][3] *= f1;
                    }
                    M0 = n0; M1 = n1;
                    thr0 = (M0 - cz0) * su; thr1 = (M1 - cz1) * su;
                    negoff = f2_pack(M0 == -INFINITY ? -INFINITY : cz0 + 12.f - M0,
                                     M1 == -INFINITY ? -INFINITY : cz1 + 12.f - M1);
                }
                #pragma unroll
                for (int gi = 0; gi < NG; ++gi) {
                    const float2 e01 = f2_unpack(f2_fma(f2_pack(T[gi][0], T[gi][1]), uu, negoff));
                    const float2 e23 = f2_unpack(f2_fma(f2_pack(T[gi][2], T[gi][3]), uu, negoff));
                    const float p0 = fast_exp2(e01.x), p1 = fast_exp2(e01.y);
                    const float p2 = fast_exp2(e23.x), p3 = fast_exp2(e23.y);
                    lsum = f2_add(lsum, f2_add(f2_pack(p0, p1), f2_pack(p2, p3)));
                    // hi parts for the columns h < 4, lo parts for the columns h + 4 (no branch:
                    // the transposes below need the whole warp converged)
                    const uint32_t hA = f2h2(p0, p1), hB = f2h2(p2, p3);
                    const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&hA));
                    const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&hB));
                    const uint32_t lA = f2h2(p0 - fa.x, p1 - fa.y), lB = f2h2(p2 - fb.x, p3 - fb.y);
                    pA[gi] = movmatrix_t((c >= 2) ? lA : hA);   // column g of tokens (c, c + 4)
                    pB[gi] = movmatrix_t((c >= 2) ? lB : hB);   // column g of tokens (c + 8, c + 12)
                }
            }
            // ---- values: 6 m-tiles (x/y of triplets 4g + m; z of 4g .. 4g + 3) ---------------
            s = slot;
            if (alive && !mbar_wait(&full[s], phase, kErrWaitFull)) alive = false;
            alive = __all_sync(0xffffffffu, alive);
            if (act && alive) {
                const uint32_t vb = smem_base + ring_off(s) + wt0 * 64 + v_lane;
                uint2 vw[NG][4];
                #pragma unroll
                for (int gi = 0; gi < NG; ++gi)
                    #pragma unroll
                    for (int t = 0; t < 4; ++t) vw[gi][t] = lds_u32x2m(vb + gi * 1024 + t * 256);   // tokens c + 4 t
                #pragma unroll
                for (int m = 0; m < 4; ++m) {
                    const uint32_t sel = (m & 1) ? 0x7624u : 0x7604u;
                    #pragma unroll
                    for (int gi = 0; gi < NG; ++gi) {
                        const uint32_t d0 = __byte_perm(pA[gi], 0u, 0x1010u), d1 = __byte_perm(pA[gi], 0u, 0x3232u);
                        const uint32_t d2 = __byte_perm(pB[gi], 0u, 0x1010u), d3 = __byte_perm(pB[gi], 0u, 0x3232u);
                        const uint2 x0 = lds_u32x2m(__byte_perm((m >> 1) ? vw[gi][0].y : vw[gi][0].x, lanereg, sel));
                        const uint2 x1 = lds_u32x2m(__byte_perm((m >> 1) ? vw[gi][1].y : vw[gi][1].x, lanereg, sel));
                        const uint2 x2 = lds_u32x2m(__byte_perm((m >> 1) ? vw[gi][2].y : vw[gi][2].x, lanereg, sel));
                        const uint2 x3 = lds_u32x2m(__byte_perm((m >> 1) ? vw[gi][3].y : vw[gi][3].x, lanereg, sel));
                        mma16816(acc[m], x0.x, x0.y, x1.x, x1.y, d0, d1);
                        mma16816(acc[m], x2.x, x2.y, x3.x, x3.y, d2, d3);
                    }
                }
                #pragma unroll
                for (int m = 0; m < 2; ++m) {
                    // i_z - 8 of two tokens' codes as exact fp16 (1024 + i_z, less 1032): centred, so
                    // that sum p (i_z - 8) does not grow tile by tile -- o_z = (z0 + 8 dz) l + dz
                    // sum p (i_z - 8) then has no cancellation for the truncating tensor-core sums
                    // to expose.  The tile's sums start from zero and join the running sums by
                    // fp32 adds.
                    float zt[4] = {0.f, 0.f, 0.f, 0.f};
                    #pragma unroll
                    for (int gi = 0; gi < NG; ++gi) {
                        const uint32_t wa = m ? vw[gi][0].y : vw[gi][0].x, wb = m ? vw[gi][1].y : vw[gi][1].x;
                        const uint32_t wc2 = m ? vw[gi][2].y : vw[gi][2].x, wd = m ? vw[gi][3].y : vw[gi][3].x;
                        mma16816(zt, zc8(prmt(wa, wb, 0x5511u)), zc8(prmt(wa, wb, 0x7733u)),
                                 zc8(prmt(wc2, wd, 0x5511u)), zc8(prmt(wc2, wd, 0x7733u)), pA[gi], pB[gi]);
                    }
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) acc[4 + m][i] += zt[i];
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++slot == SLOTS) { slot = 0; phase ^= 1u; }
        }
        {                                                  // prefetch the next item's queries
            WorkCursor pc = wc;
            ItemRange rn;
            if (tid < HQ * 96 && work_next<true>(p, pc, rn))
                qreg = q_load(p.q, p.qdt, (int64_t)rn.b * p.q_bs + (int64_t)(rn.hk * HQ + tid / 96) * p.q_hs +
                              tid % 96);
        }
        // ---- merge: hi + lo columns, the lanes of a warp, then the warps ----------------------
        float2 lsf = f2_unpack(lsum);
        #pragma unroll
        for (int off = 4; off <= 16; off <<= 1) {
            lsf.x += __shfl_xor_sync(0xffffffffu, lsf.x, off);
            lsf.y += __shfl_xor_sync(0xffffffffu, lsf.y, off);
        }
        #pragma unroll
        for (int m = 0; m < 6; ++m)
            #pragma unroll
            for (int i = 0; i < 4; ++i) acc[m][i] += __shfl_xor_sync(0xffffffffu, acc[m][i], 2);
        named_bar_sync(1, nthr);                           // every warp is done with sQ / sAcc of the last item
        if (c < 2) {
            float* o0 = sAcc + (warp * HQ + 2 * c) * 96;   // head 2c; head 2c + 1 at + 96
            #pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int t = 4 * g + m;
                o0[3 * t + 1] = acc[m][0]; o0[96 + 3 * t + 1] = acc[m][1];
                o0[3 * t + 2] = acc[m][2]; o0[96 + 3 * t + 2] = acc[m][3];
            }
            #pragma unroll
            for (int m = 0; m < 2; ++m) {
                const int t = 4 * g + 2 * m;
                o0[3 * t] = acc[4 + m][0]; o0[96 + 3 * t] = acc[4 + m][1];
                o0[3 * (t + 1)] = acc[4 + m][2]; o0[96 + 3 * (t + 1)] = acc[4 + m][3];
            }
            if (g == 0) {
                sWm[warp * HQ + 2 * c] = M0;
                sWm[warp * HQ + 2 * c + 1] = M1;
                sWl[warp * HQ + 2 * c] = lsf.x;
                sWl[warp * HQ + 2 * c + 1] = lsf.y;
            }
        }
        named_bar_sync(1, nthr);
        for (int t = tid; t < HQ * 96; t += nthr) {
            const int h = t / 96, k = t % 96;
            float M = -INFINITY;
            #pragma unroll
            for (int w = 0; w < W; ++w) M = fmaxf(M, sWm[w * HQ + h]);
            float v = 0.f, L = 0.f;
            #pragma unroll
            for (int w = 0; w < W; ++w) {
                const float mw = sWm[w * HQ + h];
                const float f = (mw == -INFINITY) ? 0.f : fast_exp2(mw - M);
                v = fmaf(f, sAcc[w * HQ * 96 + h * 96 + k], v);
                L = fmaf(f, sWl[w * HQ + h], L);
            }
            // z: sum p (z0 + dz i_z) = (z0 + 8 dz) l + dz sum p (i_z - 8)
            if (k % 3 == 0) v = fmaf(dz, v, fmaf(8.f, dz, z0) * L);
            // the weights carry 2^12 (2^12 exp2(s - M)): drop it, so that m is the running max
            sAcc[h * 96 + k] = v * 0x1p-12f;               // warp 0's block: only this thread reads it
            if (k == 0) {
                sM[h] = M;
                sL[h] = L * 0x1p-12f;
            }
        }
        named_bar_sync(1, nthr);
        finish_item(p, r, sM, sL, sAcc, sFin, sflag, p.R, 96, tid, nthr, 1);
    }
    xr_finish_call(p, sAcc, sFin, p.R, 96, tid, nthr, 1);
}

}  // namespace pkv
