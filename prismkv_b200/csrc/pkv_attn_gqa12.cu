// pkv_attn_gqa12.cu -- decode attention for grouped query heads over 12-bit (4+4+4) uniform-polar
// codes of head_dim 96.  One work unit is four query heads of one KV head, so every K and V code
// of the unit is read and decoded ONCE for the four heads (the one-head kernels decode it once
// per query head).  Query groups of 8, 12, ... heads are 2, 3, ... units over the same KV head.
//
// One CTA per SM: 19 consumer warps and one TMA producer warp (five warps per SM sub-partition
// leave 96 registers a thread).  The producer streams half tiles (the K or the V codes of 304
// tokens, 19 KB) into a ring of four slots, consumed in the order K0 V0 K1 V1 ...; a consumer
// warp owns 16 tokens of every tile.
//
//  * K (8 lanes per token, lane = (token tq, triplets 4g .. 4g+3)): a 128 KB table holds, for
//    every flat polar index e = (i_r << 4) | i_theta and triplet j, the four heads' q'_x x(e) +
//    q'_y y(e) as one float4.  The table is two halves of [256 e][16 slots]; triplet 4g + i sits
//    in half i >> 1, slot 8 (i & 1) + g, so one byte permute turns a code's flat byte into its
//    row offset e * 256 + 16 g, and the eight triplets one load instruction touches (lanes
//    g = 0..7) fall in eight distinct bank groups: four 16-byte wavefronts per warp load, the
//    minimum, for any codes.  z enters through the code bits (uniform bins are affine in i_z):
//    a byte permute builds the float 0.5 + i_z / 256 and the constant part moves into the
//    per-head score offset.  An 8-lane transpose-reduce completes 16 tokens x 4 heads; each
//    lane walks its token steps in the order it ^ (g >> 1), so that reduce needs no selects
//    over steps.
//  * softmax: per warp and head a running max (rescale only when a warp vote sees a larger
//    score); the weights go to a per-warp buffer as duplicated pairs (p, p).
//  * V (16 lanes per token, lane = (token, triplets 2c, 2c+1)): z and r from the code bits
//    under the 2^23 exponent, (cos, sin) from a 16-entry table; x, y are formed once and then
//    accumulated for the four heads with paired fp32 FMAs.
//
// Work: persistent CTAs over balanced tile ranges or round-robin items (the shared cursor of
// pkv_attn.cu); splits of a unit merge in the last CTA to finish (finish_item).  Every
// mbarrier wait is bounded: on expiry the device error word is set and the CTA stops reading.
// All arithmetic is fp32; the result equals softmax(q . decode(K)^T * scale) . decode(V)
// (polar_attention.py:277-309 with decoded values) within fp32 rounding.

namespace pkv {
namespace gqa12 {
constexpr int W = 19;                                   // consumer warps (20 warps: 96 registers)
constexpr int HQ = 4;                                   // query heads per unit
constexpr int TW = 16;                                  // tokens per warp per tile
constexpr int TT = W * TW;                              // tokens per tile
constexpr int HALF = TT * 64;                           // K (or V) codes of a tile: 32 x uint16 / token
constexpr int SLOTS = 3;                                // ring of half tiles
constexpr int KT_HALF = 256 * 16 * 16;                  // [256 flat][16 slots] float4
constexpr int KT_BYTES = 2 * KT_HALF;
constexpr int OFF_KT = 0;
constexpr int OFF_RING = OFF_KT + KT_BYTES;
constexpr int XY_COPIES = 8;                            // V's (x, y) table, one copy per 2 lane columns
constexpr int OFF_XY = OFF_RING + SLOTS * HALF;         // [256 flat][8 copies] float2: (x, y) of the flat index
constexpr int OFF_CS = OFF_XY + 256 * XY_COPIES * 8;    // [16] float2, 128-byte aligned
constexpr int OFF_Q = OFF_CS + 128;                     // [4][96] rotated, scaled queries
constexpr int OFF_QRAW = OFF_Q + HQ * 96 * 4;           // [4][96] raw queries
constexpr int OFF_P = OFF_QRAW + HQ * 96 * 4;           // [W][TW tokens][2] float4 weight pairs
constexpr int OFF_WML = OFF_P + W * TW * 2 * 16;        // [W][4] max, [W][4] sum
constexpr int OFF_FIN = OFF_WML + 2 * W * HQ * 4;       // [4][96]
constexpr int OFF_MISC = OFF_FIN + HQ * 96 * 4;         // sM[4], sL[4], sC[4], flag
constexpr int OFF_BAR = OFF_MISC + 64;                  // full[SLOTS], empty[SLOTS], rbar
constexpr int TOTAL = OFF_BAR + (2 * SLOTS + 1) * 8;
constexpr int OFF_ACC = OFF_KT;                         // item merge [W][4][96] over the dead table
constexpr int OFF_R = OFF_KT + 32768;                   // R (fp32, row pitch 96) over the dead table
constexpr int RBYTES = 96 * 96 * 4;
constexpr float MAGIC = 8388608.f;                      // 2^23
static_assert(W * HQ * 96 * 4 <= OFF_R - OFF_KT && OFF_R + RBYTES <= OFF_KT + KT_BYTES,
              "merge buffer and R fit the table region side by side");
static_assert(OFF_RING % 128 == 0 && OFF_XY % 128 == 0 && OFF_CS % 128 == 0 && OFF_P % 16 == 0 &&
              OFF_BAR % 8 == 0, "alignment");
static_assert(TOTAL <= 227 * 1024, "one CTA per SM");
static_assert(W * 32 >= HQ * 96, "one consumer thread per query element (the query prefetch)");
}  // namespace gqa12

__device__ __forceinline__ uint2 lds_u32x2(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ float4 lds_f32x4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

// Producer: half tiles in consumption order (K of tile t, then V of tile t) into the ring.
__device__ void produce_gqa12(const AttnParams& p, uint8_t* ring, uint64_t* full, uint64_t* empty) {
    using namespace gqa12;
    int seq = 0, s = 0;
    uint32_t phase = 0;                                   // phase of slot s's next fill
    bool ok = true;
    WorkCursor wc = work_begin(p);
    ItemRange r;
    while (ok && work_next<true>(p, wc, r)) {
        const int64_t base = ((int64_t)r.b * p.kv_bs + (int64_t)r.kvh * p.kv_hs) * 2;
        for (int t0 = r.tok0; t0 < r.tok1 && ok; t0 += TT) {
            const uint32_t bytes = (uint32_t)min(TT, r.tok1 - t0) * 64u;
            const int64_t off = base + (int64_t)t0 * 64;
            #pragma unroll 1
            for (int h = 0; h < 2; ++h) {
                if (seq >= SLOTS && !mbar_wait(&empty[s], phase ^ 1u, kErrWaitEmpty)) { ok = false; break; }
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s(ring + s * HALF, (h ? p.vc : p.kc) + off, bytes, &full[s]);
                ++seq;
                if (++s == SLOTS) { s = 0; phase ^= 1u; }
            }
        }
    }
    const int issued = seq;                               // drain before the CTA may exit
    for (int q = max(0, issued - SLOTS); q < issued; ++q)
        mbar_wait(&full[q % SLOTS], (q / SLOTS) & 1, kErrWaitDrain);
}

__global__ void __launch_bounds__(gqa12::W * 32 + 32, 1) attn_gqa12_kernel(AttnParams p) {
    using namespace gqa12;
    extern __shared__ __align__(128) uint8_t gqa12_smem[];
    uint8_t* smem = gqa12_smem;
    float4* kT = reinterpret_cast<float4*>(smem + OFF_KT);
    float2* vCS = reinterpret_cast<float2*>(smem + OFF_CS);
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
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* empty = full + SLOTS;
    uint64_t* rbar = empty + SLOTS;
    const float* sR = reinterpret_cast<const float*>(smem + OFF_R);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float dr = p.r_max / 15.f;
    const float z0 = __ldg(p.dec_z), dz = __ldg(p.dec_z + 1) - z0;      // uniform z bins: z = z0 + i dz

    if (tid < 16) {
        // theta_i = i / 15 * 2 pi - pi (stacked_plane.py:307), scaled so that (16 i_r) * vCS = r (cos, sin)
        const float th = (float)tid / 15.f * 6.283185307179586f - 3.141592653589793f;
        vCS[tid] = make_float2(cosf(th) * dr * 0.0625f, sinf(th) * dr * 0.0625f);
    }
    if (tid == 0) {
        for (int s = 0; s < SLOTS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        mbar_init(rbar, 1);
        fence_mbar_init();
        // R for the first item's query rotation; the table overwrites it, and every item's end
        // brings it back for the finish and the next rotation
        mbar_arrive_expect_tx(rbar, RBYTES);
        bulk_g2s(smem + OFF_R, p.R, RBYTES, rbar);
    }
    // V's (x, y) table: row e = (i_r << 4) | i_theta holds XY_COPIES copies of (16 i_r) * vCS[i_theta]
    // (the same product as the radius times the (cos, sin) table), copy k at bytes 8k of the row:
    // lanes c and c + 8 share copy c & 7, two lanes (of the two tokens a load serves) per bank pair
    {
        float2* xy = reinterpret_cast<float2*>(smem + OFF_XY);
        const float drs = dr * 0.0625f;
        for (int i = tid; i < 256 * XY_COPIES; i += blockDim.x) {
            const int e = i / XY_COPIES;
            const float th = (float)(e & 15) / 15.f * 6.283185307179586f - 3.141592653589793f;
            const float rr = (float)(e & 0xF0);
            xy[i] = make_float2(rr * (cosf(th) * drs), rr * (sinf(th) * drs));
        }
    }
    float qreg = 0.f;                                     // the first item's queries, ahead of the stream
    {
        WorkCursor pc = work_begin(p);
        ItemRange r0;
        if (tid < HQ * 96 && work_next<true>(p, pc, r0))
            qreg = q_load(p.q, p.qdt, (int64_t)r0.b * p.q_bs + (int64_t)(r0.hk * HQ + tid / 96) * p.q_hs + tid % 96);
    }
    __syncthreads();
    if (warp == W) {
        if (lane == 0) produce_gqa12(p, smem + OFF_RING, full, empty);
        return;
    }

    constexpr int nthr = W * 32;
    // K lanes: tq = token of the step (0..3), g = triplet group (triplets 4g .. 4g+3).  Steps run
    // in the lane order st = it ^ fst, so the transpose-reduce below needs no selects over steps.
    const int tq = lane >> 3, g = lane & 7, fst = g >> 1;
    // V lanes: t2 = token of the step (0..1), c = word (triplets 2c, 2c+1)
    const int t2 = lane >> 4, c = lane & 15;
    const uint32_t smem_base = (uint32_t)__cvta_generic_to_shared(smem);
    const uint32_t kt_g = 16u * g;                        // byte 0 of a table address: this lane's slot
    const uint32_t csb = smem_base + OFF_CS;
    float4* pbuf = reinterpret_cast<float4*>(smem + OFF_P) + warp * TW * 2;
    int slot = 0;                                        // ring slot of the next half tile, its fill phase
    uint32_t phase = 0;
    uint32_t rphase = 0;                                 // phase of the next R copy
    bool alive = true;
    if (!mbar_wait(rbar, rphase, kErrWaitFull)) alive = false;
    rphase ^= 1u;
    WorkCursor wc = work_begin(p);
    ItemRange r;
    while (work_next<true>(p, wc, r)) {
        const int ntok = r.tok1 - r.tok0;
        const int ntiles = (ntok + TT - 1) / TT;
        if (tid < HQ * 96) sQraw[tid] = qreg;
        named_bar_sync(1, nthr);
        // q'_h = scale log2(e) R q_h: one warp per row k, lanes over the input index; the four
        // heads' sums finish in a transpose-reduce (lane bit 4 picks heads {0,1} / {2,3}, bit 3
        // one of the pair), then a butterfly over the low three lane bits
        #pragma unroll 1
        for (int k = warp; k < 96; k += W) {
            const float* row = sR + k * 96;
            const float r0 = row[lane], r1 = row[lane + 32], r2 = row[lane + 64];
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
        // score table, two halves of [256 flat][16 slots] float4: triplet j = 4 g + i lives in half
        // i >> 1, slot 8 (i & 1) + g, so a lane's four triplets are at fixed offsets from
        // flat * 256 + 16 g and the eight lane groups of one load hit eight distinct bank groups.
        // Index t < 512 fills triplet j = t & 31, theta index e0 = t >> 5, rows e0 + 16 i_r.
        for (int t = tid; t < 512; t += nthr) {
            const int j = t & 31, e0 = t >> 5;
            const float2 cs = vCS[e0];
            float A[HQ];
            #pragma unroll
            for (int h = 0; h < HQ; ++h) A[h] = sQ[h * 96 + 3 * j + 1] * cs.x + sQ[h * 96 + 3 * j + 2] * cs.y;
            const int gj = j >> 2, ij = j & 3;
            float4* dst = reinterpret_cast<float4*>(smem + OFF_KT + (ij >> 1) * KT_HALF + 128 * (ij & 1) + 16 * gj);
            #pragma unroll 4
            for (int ir = 0; ir < 16; ++ir) {
                const float f = (float)(ir << 4);
                dst[(e0 + 16 * ir) * 16] = make_float4(f * A[0], f * A[1], f * A[2], f * A[3]);
            }
        }
        // C_h = sum_j q'_h,z,j (z0 - 128 dz): the z terms below enter as (256 dz q'_z) (0.5 + i_z / 256)
        if (warp < HQ) {
            float cz = sQ[warp * 96 + 3 * lane];
            #pragma unroll
            for (int off = 16; off >= 1; off >>= 1) cz += __shfl_xor_sync(0xffffffffu, cz, off);
            if (lane == 0) sC[warp] = cz * (z0 - 128.f * dz);
        }
        named_bar_sync(1, nthr);
        // z coefficients of this lane's K triplets, 256 dz q'_h,z,j, as head pairs
        f32x2 az01[4], az23[4];
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int j = 4 * g + i;
            az01[i] = f2_pack(sQ[0 * 96 + 3 * j] * dz * 256.f, sQ[1 * 96 + 3 * j] * dz * 256.f);
            az23[i] = f2_pack(sQ[2 * 96 + 3 * j] * dz * 256.f, sQ[3 * 96 + 3 * j] * dz * 256.f);
        }
        // after the reduce, lane (g, tq) holds token 4 fst + tq of its warp, heads 2 hp, 2 hp + 1
        const int hp = g & 1;
        const f32x2 Cp = f2_pack(sC[2 * hp], sC[2 * hp + 1]);
        const f32x2 negm = f2_pack(-MAGIC, -MAGIC);
        float2 mp = make_float2(-INFINITY, -INFINITY);      // running max of this lane's head pair
        f32x2 lsum = f2_pack(0.f, 0.f);
        f32x2 azz[HQ], axa[HQ], axb[HQ];                    // V: (z_2c, z_2c+1), (x, y)_2c, (x, y)_2c+1
        #pragma unroll
        for (int h = 0; h < HQ; ++h) {
            azz[h] = f2_pack(0.f, 0.f);
            axa[h] = f2_pack(0.f, 0.f);
            axb[h] = f2_pack(0.f, 0.f);
        }

        for (int tile = 0; tile < ntiles; ++tile) {
            const int nt = min(TT, ntok - tile * TT);
            const int wt0 = warp * TW;                      // this warp's first token of the tile
            // ---- K: scores of 16 tokens x 4 heads ----------------------------------------
            int s = slot;
            if (alive && !mbar_wait(&full[s], phase, kErrWaitFull)) alive = false;
            const bool act = alive && wt0 < nt;
            float2 sc = make_float2(-INFINITY, -INFINITY);
            if (act) {
                // token-step it ^ fst of this lane: within the warp's 1 KB of the tile the step
                // offset 256 (it ^ fst) is an XOR into offset bits 8-9
                const uint32_t kslot = smem_base + OFF_RING + s * HALF + wt0 * 64;
                const uint32_t kofs = (tq * 64 + g * 8) | (fst << 8);
                const uint32_t ktab = smem_base + OFF_KT;
                f32x2 v01[4], v23[4];
                #pragma unroll
                for (int it = 0; it < 4; ++it) {
                    const uint2 cw = lds_u32x2(kslot + (kofs ^ (it << 8)));
                    f32x2 s01, s23;
                    #pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const uint32_t w = u ? cw.y : cw.x;
                        // flat * 256 + 16 g from one byte permute (byte 0 from the lane's slot)
                        const uint32_t ea = __byte_perm(w, kt_g, 0x5504), eb = __byte_perm(w, kt_g, 0x5524);
                        f32x2 ta01, ta23, tb01, tb23;
                        lds_f2x2(ktab + u * KT_HALF + ea, ta01, ta23);
                        lds_f2x2(ktab + u * KT_HALF + 128 + eb, tb01, tb23);
                        // (0.5 + i_z / 256) twice, from the byte holding i_z (two selectors that
                        // pick the same bytes, so that the pair is two independent permutes)
                        const f32x2 za = f2_pack(__int_as_float(__byte_perm(w, 0x3F000000u, 0x7144)),
                                                 __int_as_float(__byte_perm(w, 0x3F000000u, 0x7155)));
                        const f32x2 zb = f2_pack(__int_as_float(__byte_perm(w, 0x3F000000u, 0x7344)),
                                                 __int_as_float(__byte_perm(w, 0x3F000000u, 0x7355)));
                        const f32x2 t01 = f2_fma(az01[2 * u + 1], zb, f2_fma(az01[2 * u], za, f2_add(ta01, tb01)));
                        const f32x2 t23 = f2_fma(az23[2 * u + 1], zb, f2_fma(az23[2 * u], za, f2_add(ta23, tb23)));
                        s01 = u ? f2_add(s01, t01) : t01;
                        s23 = u ? f2_add(s23, t23) : t23;
                    }
                    v01[it] = s01;
                    v23[it] = s23;
                }
                // 8-lane transpose-reduce of (step, head): lane bit 2 keeps iterations {0,1} and
                // bit 1 iteration 0 -- the same token-step fst on both sides of each exchange --
                // then bit 0 the head pair
                #pragma unroll
                for (int it = 0; it < 2; ++it) {
                    const float2 a01 = f2_unpack(v01[it + 2]), a23 = f2_unpack(v23[it + 2]);
                    v01[it] = f2_add(v01[it], f2_pack(__shfl_xor_sync(0xffffffffu, a01.x, 4),
                                                      __shfl_xor_sync(0xffffffffu, a01.y, 4)));
                    v23[it] = f2_add(v23[it], f2_pack(__shfl_xor_sync(0xffffffffu, a23.x, 4),
                                                      __shfl_xor_sync(0xffffffffu, a23.y, 4)));
                }
                {
                    const float2 a01 = f2_unpack(v01[1]), a23 = f2_unpack(v23[1]);
                    v01[0] = f2_add(v01[0], f2_pack(__shfl_xor_sync(0xffffffffu, a01.x, 2),
                                                    __shfl_xor_sync(0xffffffffu, a01.y, 2)));
                    v23[0] = f2_add(v23[0], f2_pack(__shfl_xor_sync(0xffffffffu, a23.x, 2),
                                                    __shfl_xor_sync(0xffffffffu, a23.y, 2)));
                }
                {
                    const f32x2 keep = hp ? v23[0] : v01[0], send = hp ? v01[0] : v23[0];
                    const float2 sd = f2_unpack(send);
                    sc = f2_unpack(f2_add(f2_add(keep, f2_pack(__shfl_xor_sync(0xffffffffu, sd.x, 1),
                                                              __shfl_xor_sync(0xffffffffu, sd.y, 1))), Cp));
                }
                if (wt0 + 4 * fst + tq >= nt) sc = make_float2(-INFINITY, -INFINITY);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++slot == SLOTS) { slot = 0; phase ^= 1u; }
            // ---- online softmax per head ------------------------------------------------
            if (act) {
                if (__any_sync(0xffffffffu, sc.x > mp.x || sc.y > mp.y)) {      // rare after the first tiles
                    float2 mt = sc;
                    #pragma unroll
                    for (int off = 2; off <= 16; off <<= 1) {
                        mt.x = fmaxf(mt.x, __shfl_xor_sync(0xffffffffu, mt.x, off));
                        mt.y = fmaxf(mt.y, __shfl_xor_sync(0xffffffffu, mt.y, off));
                    }
                    const float2 mn = make_float2(fmaxf(mp.x, mt.x), fmaxf(mp.y, mt.y));
                    const float2 f = make_float2(fast_exp2(mp.x - mn.x), fast_exp2(mp.y - mn.y));  // 0 from -inf
                    const float2 fo = make_float2(__shfl_xor_sync(0xffffffffu, f.x, 1),
                                                  __shfl_xor_sync(0xffffffffu, f.y, 1));
                    const float f4[HQ] = {hp ? fo.x : f.x, hp ? fo.y : f.y, hp ? f.x : fo.x, hp ? f.y : fo.y};
                    lsum = f2_mul(lsum, f2_pack(f.x, f.y));
                    #pragma unroll
                    for (int h = 0; h < HQ; ++h) {
                        const f32x2 ff = f2_pack(f4[h], f4[h]);
                        azz[h] = f2_mul(azz[h], ff);
                        axa[h] = f2_mul(axa[h], ff);
                        axb[h] = f2_mul(axb[h], ff);
                    }
                    mp = mn;
                }
                const float px = (mp.x == -INFINITY) ? 0.f : fast_exp2(sc.x - mp.x);
                const float py = (mp.y == -INFINITY) ? 0.f : fast_exp2(sc.y - mp.y);
                lsum = f2_add(lsum, f2_pack(px, py));
                pbuf[(4 * fst + tq) * 2 + hp] = make_float4(px, px, py, py);
            }
            __syncwarp();
            // ---- V: weighted sums of 16 tokens for 4 heads -------------------------------
            s = slot;
            if (alive && !mbar_wait(&full[s], phase, kErrWaitFull)) alive = false;
            if (act && alive) {
                const uint32_t vh = smem_base + OFF_RING + s * HALF + wt0 * 64 + t2 * 64 + c * 4;
                const uint32_t pb = smem_base + OFF_P + warp * TW * 32 + t2 * 32;
                const uint32_t xyl = smem_base + OFF_XY + (c & (XY_COPIES - 1)) * 8;
                #pragma unroll 4
                for (int st = 0; st < TW / 2; ++st) {
                    const uint32_t w = lds_u32(vh + st * 128);
                    f32x2 pp[HQ];                                   // (p_h, p_h) of the step's token
                    lds_f2x2(pb + st * 64, pp[0], pp[1]);
                    lds_f2x2(pb + st * 64 + 16, pp[2], pp[3]);
                    const f32x2 zz = f2_add(f2_pack(__int_as_float(__byte_perm(w, 0x4B000000u, 0x7514)),
                                                    __int_as_float(__byte_perm(w, 0x4B000000u, 0x7534))), negm);
                    // (x, y) of both codes from the flat bytes 0 and 2: row e at e * 64, this lane's copy
                    const f32x2 xa = lds_f2(xyl + __byte_perm(w, 0u, 0x4440) * 64u);
                    const f32x2 xb = lds_f2(xyl + __byte_perm(w, 0u, 0x4442) * 64u);
                    #pragma unroll
                    for (int h = 0; h < HQ; ++h) {
                        azz[h] = f2_fma(pp[h], zz, azz[h]);
                        axa[h] = f2_fma(pp[h], xa, axa[h]);
                        axb[h] = f2_fma(pp[h], xb, axb[h]);
                    }
                }
            }
            __syncwarp();                                   // pbuf is rewritten by the next tile
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
        // ---- merge: lanes of a warp, then the warps -----------------------------------------
        float2 lsf = f2_unpack(lsum);
        #pragma unroll
        for (int off = 2; off <= 16; off <<= 1) {
            lsf.x += __shfl_xor_sync(0xffffffffu, lsf.x, off);
            lsf.y += __shfl_xor_sync(0xffffffffu, lsf.y, off);
        }
        float2 vz[HQ], va[HQ], vb[HQ];
        #pragma unroll
        for (int h = 0; h < HQ; ++h) {
            vz[h] = f2_unpack(azz[h]);
            va[h] = f2_unpack(axa[h]);
            vb[h] = f2_unpack(axb[h]);
            vz[h].x += __shfl_xor_sync(0xffffffffu, vz[h].x, 16);
            vz[h].y += __shfl_xor_sync(0xffffffffu, vz[h].y, 16);
            va[h].x += __shfl_xor_sync(0xffffffffu, va[h].x, 16);
            va[h].y += __shfl_xor_sync(0xffffffffu, va[h].y, 16);
            vb[h].x += __shfl_xor_sync(0xffffffffu, vb[h].x, 16);
            vb[h].y += __shfl_xor_sync(0xffffffffu, vb[h].y, 16);
        }
        named_bar_sync(1, nthr);                           // every warp is past its last table read
        if (tid == 0) {                                    // R over the dead table, beside the merge buffer
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(rbar, RBYTES);
            bulk_g2s(smem + OFF_R, p.R, RBYTES, rbar);
        }
        if (lane < 16) {
            float* o = sAcc + warp * HQ * 96 + 6 * c;      // triplets 2c, 2c + 1
            #pragma unroll
            for (int h = 0; h < HQ; ++h) {
                o[h * 96 + 0] = vz[h].x; o[h * 96 + 1] = va[h].x; o[h * 96 + 2] = va[h].y;
                o[h * 96 + 3] = vz[h].y; o[h * 96 + 4] = vb[h].x; o[h * 96 + 5] = vb[h].y;
            }
        }
        if (lane < 2) {
            sWm[warp * HQ + 2 * lane] = mp.x;
            sWm[warp * HQ + 2 * lane + 1] = mp.y;
            sWl[warp * HQ + 2 * lane] = lsf.x;
            sWl[warp * HQ + 2 * lane + 1] = lsf.y;
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
            // z: sum p (z0 + dz i_z) = z0 l + dz/256 * sum p (256 i_z)
            if (k % 3 == 0) v = fmaf(dz * (1.f / 256.f), v, z0 * L);
            sAcc[h * 96 + k] = v;                          // warp 0's block: only this thread reads it
            if (k == 0) {
                sM[h] = M;
                sL[h] = L;
            }
        }
        if (alive && !mbar_wait(rbar, rphase, kErrWaitFull)) alive = false;
        rphase ^= 1u;
        named_bar_sync(1, nthr);
        finish_item(p, r, sM, sL, sAcc, sFin, sflag, sR, 96, tid, nthr, 1);
    }
    xr_finish_call(p, sAcc, sFin, sR, 96, tid, nthr, 1);
}

}  // namespace pkv
