// pkv_attn_mha12.cu -- decode attention for the 12-bit (4+4+4) uniform-polar, head_dim 96
// case, one query head per work unit (MHA, or grouped heads with every query head its own
// unit reading its KV head; the group's re-reads of the same codes hit L2).  Both kernels
// run two CTAs per SM of 8 consumer warps and one TMA producer warp, 256-token tiles, 32
// tokens of every tile per consumer warp, and lay their hot loops out for the shared-memory
// data path (one 128-byte wavefront per clock per SM):
//  * K: lane l reads one 32-bit word = the codes of triplets 2(l%16), 2(l%16)+1 of token
//    2s + l/16, so one warp load covers two tokens (128 bytes).  The score table row e
//    (the flat polar index) holds, in word w < 16, q'_(2w) . (x, y)(e) and in word 16 + w,
//    q'_(2w+1) . (x, y)(e); lanes of the upper half take their odd triplet first, so both
//    lookups of a step hit 32 distinct banks.  z enters through the code bits themselves
//    (uniform bins are affine in i_z): byte permutes put them under the 2^23 float
//    exponent.  A 16-lane transpose-reduce completes 32 scores per 16 steps.
//  * V: lane l reads 16 bytes = 8 codes of token l/4 (triplets 8(l%4)..+7), one warp load
//    covers 8 tokens; z and r come from the code bits, (cos, sin) from a 16-entry table
//    (one wavefront for any pattern of a half-warp).
//
// attn_mha12_kernel: two passes per item (K -> scores in shared memory, exact max, then V
// with fixed weights), items of at most 4096 tokens; R sits in shared memory, where the
// score table overlays it during the K pass.  Serves sequences of one item per unit.
//
// attn_mha12_stream_kernel: one pass with a per-warp online softmax (rescaled only when a
// warp vote sees a score above the running max) and no cap on the tokens of an item; K
// and V codes of a tile share one ring stage.  The warps' states merge once per item, then
// finish_item normalises and applies R, read from global memory (L2-resident) for the
// query rotation and the finish.  Serves longer sequences, where the two-pass kernel's
// per-item cost (R reload, score pass, weights) would recur every 4096 tokens.
//
// Every mbarrier wait is bounded (device error word on expiry, control flow kept).

namespace pkv {
namespace mha12s {
constexpr int W = 8;                                   // consumer warps
constexpr int TT = 32 * W;                             // tokens per tile (32 per warp)
constexpr int STAGES = 2;
constexpr int TILE = TT * 64;                          // K (or V) codes of a tile: 32 x uint16 per token
constexpr int STAGE = 2 * TILE;                        // K then V
constexpr int OFF_STAGE = 0;
constexpr int OFF_KT = OFF_STAGE + STAGES * STAGE;     // [256][32] score table
constexpr int OFF_CS = OFF_KT + 256 * 32 * 4;          // [16] float2 (128-byte aligned)
constexpr int OFF_Q = OFF_CS + 128;                    // [96] rotated query
constexpr int OFF_QRAW = OFF_Q + 96 * 4;               // [96] raw query
constexpr int OFF_ACC = OFF_QRAW + 96 * 4;             // [W][96] per-warp accumulators
constexpr int OFF_FIN = OFF_ACC + W * 96 * 4;          // [96]
constexpr int OFF_WML = OFF_FIN + 96 * 4;              // [W] max, [W] sum
constexpr int OFF_MISC = OFF_WML + 2 * W * 4;          // sM, sL, C, flag
constexpr int OFF_BAR = OFF_MISC + 16;                 // full[STAGES], empty[STAGES]
constexpr int TOTAL = OFF_BAR + 2 * STAGES * 8;
constexpr float MAGIC = 8388608.f;                     // 2^23
static_assert(OFF_KT % 128 == 0 && OFF_CS % 128 == 0 && OFF_BAR % 8 == 0, "alignment");
static_assert(2 * (TOTAL + 1024) <= 228 * 1024, "two CTAs per SM");
}  // namespace mha12s

// 16-lane transpose-reduce within each half-warp: on exit v[0] of lane l holds the sum over
// the 16 lanes of its half of their v[l % 16].
__device__ __forceinline__ void transpose_reduce16(float (&v)[16], int lane) {
    #pragma unroll
    for (int off = 8; off >= 1; off >>= 1) {
        const bool upper = (lane & off) != 0;
        #pragma unroll
        for (int i = 0; i < off; ++i) {
            float send = upper ? v[i] : v[i + off];
            float keep = upper ? v[i + off] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
}

// ---------------------------------------------------------------------------
// attn_mha12_kernel (two passes)
// ---------------------------------------------------------------------------
namespace mha12 {
constexpr int W = 8;                                   // consumer warps
constexpr int TT = 256;                                // tokens per tile (32 per warp)
constexpr int CH = 4096;                               // tokens per item (scores in smem)
constexpr int STAGES = 3;
constexpr int TILE = TT * 64;                          // 32 codes x 2 bytes per token
constexpr int RBYTES = 96 * 96 * 4;                    // the rotation, fp32, row pitch 96
constexpr int OFF_RT = STAGES * TILE;                  // R, or the [256][32] score table
constexpr int OFF_CS = OFF_RT + RBYTES;                // [16] float2
constexpr int OFF_Q = OFF_CS + 16 * 8;                 // [96] rotated query
constexpr int OFF_QRAW = OFF_Q + 96 * 4;               // [96] raw query
constexpr int OFF_S = OFF_QRAW + 96 * 4;               // [CH]
constexpr int OFF_RED = OFF_S + CH * 4;                // [2][W]
constexpr int OFF_ACC = OFF_RED + 2 * W * 4;           // [W][96]
constexpr int OFF_FIN = OFF_ACC + W * 96 * 4;          // [96]
constexpr int OFF_MISC = OFF_FIN + 96 * 4;             // sM, sL, C, flag
constexpr int OFF_BAR = OFF_MISC + 64;                 // full[STAGES], empty[STAGES], rbar
constexpr int TOTAL = OFF_BAR + (2 * STAGES + 1) * 8;
constexpr float MAGIC = 8388608.f;                     // 2^23
static_assert(256 * 32 * 4 <= RBYTES, "score table must fit the R region");
}  // namespace mha12


__global__ void __launch_bounds__(mha12::W * 32 + 32, 2) attn_mha12_kernel(AttnParams p) {
    using namespace mha12;
    extern __shared__ __align__(128) uint8_t mha12_smem[];
    uint8_t* smem = mha12_smem;
    float* kT = reinterpret_cast<float*>(smem + OFF_RT);       // score table, or R between uses
    const float* sR = kT;
    float2* vCS = reinterpret_cast<float2*>(smem + OFF_CS);
    float* sQ = reinterpret_cast<float*>(smem + OFF_Q);
    float* sQraw = reinterpret_cast<float*>(smem + OFF_QRAW);
    float* sS = reinterpret_cast<float*>(smem + OFF_S);
    float* sRed = reinterpret_cast<float*>(smem + OFF_RED);
    float* sAcc = reinterpret_cast<float*>(smem + OFF_ACC);
    float* sFin = reinterpret_cast<float*>(smem + OFF_FIN);
    float* sM = reinterpret_cast<float*>(smem + OFF_MISC);
    float* sL = sM + 1;
    float* sC = sM + 2;
    int* sflag = reinterpret_cast<int*>(sM + 3);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* empty = full + STAGES;
    uint64_t* rbar = empty + STAGES;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float dr = p.r_max / 15.f;
    const float z0 = __ldg(p.dec_z), dz = __ldg(p.dec_z + 1) - z0;     // uniform z bins: z = z0 + i dz

    if (tid < 16) {
        // theta_i = i / 15 * 2 pi - pi (stacked_plane.py:307), scaled so that (i_r << 4) * vCS = r (cos, sin)
        const float th = (float)tid / 15.f * 6.283185307179586f - 3.141592653589793f;
        vCS[tid] = make_float2(cosf(th) * dr * 0.0625f, sinf(th) * dr * 0.0625f);
    }
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        mbar_init(rbar, 1);
        fence_mbar_init();
        // R for the first item's query rotation, ahead of the code stream
        mbar_arrive_expect_tx(rbar, RBYTES);
        bulk_g2s(kT, p.R, RBYTES, rbar);
    }
    // the first item's query, ahead of the code stream too
    float qreg = 0.f;
    {
        WorkCursor pc = work_begin(p);
        ItemRange r0;
        if (tid < 96 && work_next<false>(p, pc, r0))
            qreg = q_load(p.q, p.qdt, (int64_t)r0.b * p.q_bs + (int64_t)r0.hk * p.q_hs + tid);
    }
    __syncthreads();
    if (warp == W) {
        if (lane == 0) produce<TT, false, false>(p, smem, TILE, full, empty, W, 2);
        return;
    }

    constexpr int nthr = W * 32;
    const int half = lane >> 4, l16 = lane & 15;
    const int wcol1 = lane, wcol2 = lane ^ 16;           // table words of the first / second code
    const int tg = lane >> 2, q4 = lane & 3;             // V: token-in-8, 8-triplet chunk
    int seq = 0, ruse = 0;
    bool alive = true;
    WorkCursor wc = work_begin(p);
    ItemRange r;
    while (work_next<false>(p, wc, r)) {
        const int ntok = r.tok1 - r.tok0;
        const int ntiles = (ntok + TT - 1) / TT;
        if (tid < 96) sQraw[tid] = qreg;
        if (alive && !mbar_wait(rbar, ruse & 1, kErrWaitFull)) alive = false;   // R in place
        named_bar_sync(1, nthr);
        // q' = scale log2(e) R q: one warp per row, lanes over the input index
        {
            const float qa = sQraw[lane], qb = sQraw[lane + 32], qc = sQraw[lane + 64];
            #pragma unroll 4
            for (int k = warp; k < 96; k += W) {
                const float* row = sR + k * 96;
                float acc = fmaf(qa, row[lane], fmaf(qb, row[lane + 32], qc * row[lane + 64]));
                #pragma unroll
                for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
                if (lane == 0) sQ[k] = acc * p.scale_log2;
            }
        }
        named_bar_sync(1, nthr);
        // score table over the R region: row e = (i_r << 4) | i_theta; word w < 16 -> triplet 2w,
        // w >= 16 -> 2(w-16)+1.  Thread t fills column t & 31, rows (t >> 5) + 8k.
        {
            const int w = tid & 31, e0 = tid >> 5;
            const int j = (w < 16) ? 2 * w : 2 * (w - 16) + 1;
            const float qx = sQ[3 * j + 1], qy = sQ[3 * j + 2];
            const float2 cs0 = vCS[e0 & 15], cs1 = vCS[(e0 + 8) & 15];
            const float A0 = qx * cs0.x + qy * cs0.y, A1 = qx * cs1.x + qy * cs1.y;
            #pragma unroll 8
            for (int k = 0; k < 32; ++k) {
                const int e = e0 + 8 * k;
                kT[e * 32 + w] = (float)(e & 0xF0) * ((k & 1) ? A1 : A0);
            }
        }
        if (warp == 0) {                                   // C = z0 * sum_j q'_z,j
            float c = sQ[3 * lane];
            #pragma unroll
            for (int off = 16; off >= 1; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
            if (lane == 0) sC[0] = c * z0;
        }
        named_bar_sync(1, nthr);
        // z coefficient per code of this lane: q'_z,j * dz / 256 (the code bits give 256 i_z)
        const int j1 = 2 * l16 + half, j2 = 2 * l16 + 1 - half;
        const float2 az = make_float2(sQ[3 * j1] * dz * (1.f / 256.f), sQ[3 * j2] * dz * (1.f / 256.f));
        const float C = sC[0];
        const uint32_t kb1 = (uint32_t)__cvta_generic_to_shared(kT) + 4u * wcol1;   // this lane's table words
        const uint32_t kb2 = (uint32_t)__cvta_generic_to_shared(kT) + 4u * wcol2;
        // byte selectors: a word holds two 12-bit codes, the first in bytes 0-1.  selr* pull the
        // low byte (the flat polar index); selz* put byte 1 (z in its low nibble) under the
        // 2^23 exponent, giving 2^23 + 256 i_z.  Half 1 of the warp takes the codes swapped.
        const uint32_t selr1 = half ? 0x4442u : 0x4440u, selr2 = half ? 0x4440u : 0x4442u;
        const uint32_t selz1 = half ? 0x7534u : 0x7514u, selz2 = half ? 0x7514u : 0x7534u;

        // ---- pass 1: K -> scores ------------------------------------------------
        float mx = -INFINITY;
        for (int tile = 0; tile < ntiles; ++tile, ++seq) {
            const int s = seq % STAGES;
            if (alive && !mbar_wait(&full[s], (seq / STAGES) & 1, kErrWaitFull)) alive = false;
            const uint32_t* K32 = reinterpret_cast<const uint32_t*>(smem + s * TILE);
            const int nt = min(TT, ntok - tile * TT);
            if (alive && warp * 32 < nt) {
                float ps[16];
                #pragma unroll
                for (int st = 0; st < 16; ++st) {
                    const uint32_t w = K32[(warp * 32 + 2 * st + half) * 16 + l16];
                    const uint32_t i1 = __byte_perm(w, 0u, selr1), i2 = __byte_perm(w, 0u, selr2);
                    const float2 zz = fadd2(make_float2(__int_as_float(__byte_perm(w, 0x4B000000u, selz1)),
                                                        __int_as_float(__byte_perm(w, 0x4B000000u, selz2))),
                                            make_float2(-MAGIC, -MAGIC));
                    const float t1 = lds_f32(kb1 + i1 * 128u);
                    const float t2 = lds_f32(kb2 + i2 * 128u);
                    const float2 a = ffma2(az, zz, make_float2(t1, t2));
                    ps[st] = a.x + a.y;
                }
                transpose_reduce16(ps, lane);
                const int tok = warp * 32 + 2 * l16 + half;
                if (tok < nt) {
                    const float sc = ps[0] + C;
                    sS[tile * TT + tok] = sc;
                    mx = fmaxf(mx, sc);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        #pragma unroll
        for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        if (lane == 0) sRed[warp] = mx;
        named_bar_sync(1, nthr);
        // the score table is dead: bring R back for the finish and the next rotation
        if (tid == 0) {
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(rbar, RBYTES);
            bulk_g2s(kT, p.R, RBYTES, rbar);
        }
        ++ruse;
        // prefetch the next item's query
        {
            WorkCursor pc = wc;
            ItemRange rn;
            if (tid < 96 && work_next<false>(p, pc, rn))
                qreg = q_load(p.q, p.qdt, (int64_t)rn.b * p.q_bs + (int64_t)rn.hk * p.q_hs + tid);
        }
        float M = -INFINITY;
        #pragma unroll
        for (int w = 0; w < W; ++w) M = fmaxf(M, sRed[w]);
        // ---- weights ------------------------------------------------------------
        float lp = 0.f;
        for (int t = tid; t < ntiles * TT; t += nthr) {
            const float pv = (t < ntok && M != -INFINITY) ? fast_exp2(sS[t] - M) : 0.f;
            sS[t] = pv;
            lp += pv;
        }
        #pragma unroll
        for (int off = 16; off >= 1; off >>= 1) lp += __shfl_xor_sync(0xffffffffu, lp, off);
        if (lane == 0) sRed[W + warp] = lp;
        named_bar_sync(1, nthr);
        if (tid == 0) {
            float l = 0.f;
            for (int w = 0; w < W; ++w) l += sRed[W + w];
            sL[0] = l;
            sM[0] = M;
        }

        // ---- pass 2: V with fixed weights ---------------------------------------
        float2 axy[8], azz[4];
        #pragma unroll
        for (int k = 0; k < 8; ++k) axy[k] = make_float2(0.f, 0.f);
        #pragma unroll
        for (int k = 0; k < 4; ++k) azz[k] = make_float2(0.f, 0.f);
        const uint32_t csb = (uint32_t)__cvta_generic_to_shared(vCS);
        for (int tile = 0; tile < ntiles; ++tile, ++seq) {
            const int s = seq % STAGES;
            if (alive && !mbar_wait(&full[s], (seq / STAGES) & 1, kErrWaitFull)) alive = false;
            const uint4* V16 = reinterpret_cast<const uint4*>(smem + s * TILE);
            const int nt = min(TT, ntok - tile * TT);
            if (alive && warp * 32 < nt) {
                #pragma unroll
                for (int st = 0; st < 4; ++st) {
                    const int tok = warp * 32 + 8 * st + tg;
                    const uint4 wv = V16[tok * 4 + q4];
                    const float pw = sS[tile * TT + tok];
                    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
                    #pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        const uint32_t w = ww[h];
                        // low code (triplet 8 q4 + 2h), high code (8 q4 + 2h + 1)
                        const float2 zf = fadd2(make_float2(__int_as_float((w & 0xF00u) | 0x4B000000u),
                                                            __int_as_float(__byte_perm(w, 0x4B000000u, 0x7534))),
                                                make_float2(-MAGIC, -MAGIC));
                        const float2 rf = fadd2(make_float2(__int_as_float((w & 0xF0u) | 0x4B000000u),
                                                            __int_as_float(((w >> 16) & 0xF0u) | 0x4B000000u)),
                                                make_float2(-MAGIC, -MAGIC));
                        const float2 cs0 = lds_f32x2(csb | ((w << 3) & 0x78u));      // table is 128-byte aligned
                        const float2 cs1 = lds_f32x2(csb | ((w >> 13) & 0x78u));
                        azz[h] = ffma2(make_float2(pw, pw), zf, azz[h]);
                        const float2 wr = fmul2(make_float2(pw, pw), rf);
                        axy[2 * h] = ffma2(make_float2(wr.x, wr.x), cs0, axy[2 * h]);
                        axy[2 * h + 1] = ffma2(make_float2(wr.y, wr.y), cs1, axy[2 * h + 1]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // reduce over the 8 token groups of the warp (lanes sharing q4)
        #pragma unroll
        for (int off = 4; off <= 16; off <<= 1) {
            #pragma unroll
            for (int k = 0; k < 8; ++k) {
                axy[k].x += __shfl_xor_sync(0xffffffffu, axy[k].x, off);
                axy[k].y += __shfl_xor_sync(0xffffffffu, axy[k].y, off);
            }
            #pragma unroll
            for (int k = 0; k < 4; ++k) {
                azz[k].x += __shfl_xor_sync(0xffffffffu, azz[k].x, off);
                azz[k].y += __shfl_xor_sync(0xffffffffu, azz[k].y, off);
            }
        }
        if (tg == 0) {
            float* o = sAcc + warp * 96 + 24 * q4;          // triplets 8 q4 .. 8 q4 + 7
            #pragma unroll
            for (int h = 0; h < 4; ++h) {
                o[6 * h + 0] = azz[h].x;  o[6 * h + 1] = axy[2 * h].x;      o[6 * h + 2] = axy[2 * h].y;
                o[6 * h + 3] = azz[h].y;  o[6 * h + 4] = axy[2 * h + 1].x;  o[6 * h + 5] = axy[2 * h + 1].y;
            }
        }
        named_bar_sync(1, nthr);
        if (tid < 96) {
            float v = 0.f;
            #pragma unroll
            for (int w = 0; w < W; ++w) v += sAcc[w * 96 + tid];
            // z: sum p (z0 + dz i_z) = z0 l + dz/256 * sum p (256 i_z)
            if (tid % 3 == 0) v = fmaf(z0, sL[0], v * dz * (1.f / 256.f));
            sAcc[tid] = v;
        }
        if (alive && !mbar_wait(rbar, ruse & 1, kErrWaitFull)) alive = false;   // R back in place
        named_bar_sync(1, nthr);
        finish_item(p, r, sM, sL, sAcc, sFin, sflag, sR, 96, tid, nthr, 1);
    }
    xr_finish_call(p, sAcc, sFin, sR, 96, tid, nthr, 1);
    // the last R copy must land before the CTA exits
    if (tid == 0 && alive) mbar_wait(rbar, ruse & 1, kErrWaitDrain);
}


// ---------------------------------------------------------------------------
// attn_mha12_stream_kernel (one pass)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(mha12s::W * 32 + 32, 2) attn_mha12_stream_kernel(AttnParams p) {
    using namespace mha12s;
    extern __shared__ __align__(128) uint8_t mha12s_smem[];
    uint8_t* smem = mha12s_smem;
    float* kT = reinterpret_cast<float*>(smem + OFF_KT);       // score table
    float2* vCS = reinterpret_cast<float2*>(smem + OFF_CS);
    float* sQ = reinterpret_cast<float*>(smem + OFF_Q);
    float* sQraw = reinterpret_cast<float*>(smem + OFF_QRAW);
    float* sAcc = reinterpret_cast<float*>(smem + OFF_ACC);
    float* sFin = reinterpret_cast<float*>(smem + OFF_FIN);
    float* sWm = reinterpret_cast<float*>(smem + OFF_WML);
    float* sWl = sWm + W;
    float* sM = reinterpret_cast<float*>(smem + OFF_MISC);
    float* sL = sM + 1;
    float* sC = sM + 2;
    int* sflag = reinterpret_cast<int*>(sM + 3);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* empty = full + STAGES;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // R (36 KB) is read from global memory by every item's rotation and finish; once the code
    // stream runs, a miss on it waits behind the bulk copies, so bring it into L2 first
    constexpr int R_LINES = 96 * 96 * 4 / 128;
    for (int i = tid; i < R_LINES; i += blockDim.x) prefetch_l2(p.R + i * 32);
    const float dr = p.r_max / 15.f;
    const float z0 = __ldg(p.dec_z), dz = __ldg(p.dec_z + 1) - z0;     // uniform z bins: z = z0 + i dz

    if (tid < 16) {
        // theta_i = i / 15 * 2 pi - pi (stacked_plane.py:307), scaled so that (i_r << 4) * vCS = r (cos, sin)
        const float th = (float)tid / 15.f * 6.283185307179586f - 3.141592653589793f;
        vCS[tid] = make_float2(cosf(th) * dr * 0.0625f, sinf(th) * dr * 0.0625f);
    }
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        fence_mbar_init();
    }
    float qreg = 0.f;                      // the first item's query, ahead of the code stream too
    {
        WorkCursor pc = work_begin(p);
        ItemRange r0;
        if (tid < 96 && work_next<false>(p, pc, r0))
            qreg = q_load(p.q, p.qdt, (int64_t)r0.b * p.q_bs + (int64_t)r0.hk * p.q_hs + tid);
    }
    __syncthreads();
    if (warp == W) {
        if (lane == 0) produce<TT, true, false>(p, smem + OFF_STAGE, STAGE, full, empty, W, 2);
        return;
    }

    constexpr int nthr = W * 32;
    const int half = lane >> 4, l16 = lane & 15;
    const int tg = lane >> 2, q4 = lane & 3;             // V: token-in-8, 8-triplet chunk
    const uint32_t kb1 = (uint32_t)__cvta_generic_to_shared(kT) + 4u * lane;          // table words of the
    const uint32_t kb2 = (uint32_t)__cvta_generic_to_shared(kT) + 4u * (lane ^ 16);   // first / second code
    const uint32_t csb = (uint32_t)__cvta_generic_to_shared(vCS);
    // byte selectors: a word holds two 12-bit codes, the first in bytes 0-1.  selr* pull the
    // low byte (the flat polar index); selz* put byte 1 (z in its low nibble) under the
    // 2^23 exponent, giving 2^23 + 256 i_z.  Half 1 of the warp takes the codes swapped.
    const uint32_t selr1 = half ? 0x4442u : 0x4440u, selr2 = half ? 0x4440u : 0x4442u;
    const uint32_t selz1 = half ? 0x7534u : 0x7514u, selz2 = half ? 0x7514u : 0x7534u;
    int seq = 0;
    bool alive = true;
    WorkCursor wc = work_begin(p);
    ItemRange r;
    while (work_next<false>(p, wc, r)) {
        const int ntok = r.tok1 - r.tok0;
        const int ntiles = (ntok + TT - 1) / TT;
        if (tid < 96) sQraw[tid] = qreg;
        named_bar_sync(1, nthr);
        // q' = scale log2(e) R q: one warp per row, lanes over the input index (R from L2)
        {
            const float qa = sQraw[lane], qb = sQraw[lane + 32], qc = sQraw[lane + 64];
            #pragma unroll 4
            for (int k = warp; k < 96; k += W) {
                const float* row = p.R + k * 96;
                float acc = fmaf(qa, __ldg(row + lane), fmaf(qb, __ldg(row + lane + 32), qc * __ldg(row + lane + 64)));
                #pragma unroll
                for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
                if (lane == 0) sQ[k] = acc * p.scale_log2;
            }
        }
        named_bar_sync(1, nthr);
        // score table: row e = (i_r << 4) | i_theta; word w < 16 -> triplet 2w, w >= 16 ->
        // 2(w-16)+1.  Warp v fills rows v + 8k (theta index v, then v + 8), lane w column w.
        // The previous item's last table reads are behind the barriers above.
        {
            const int j = (lane < 16) ? 2 * lane : 2 * (lane - 16) + 1;
            const float qx = sQ[3 * j + 1], qy = sQ[3 * j + 2];
            const float2 cs0 = vCS[warp], cs1 = vCS[warp + 8];
            const float A0 = qx * cs0.x + qy * cs0.y, A1 = qx * cs1.x + qy * cs1.y;
            #pragma unroll 8
            for (int k = 0; k < 32; ++k) {
                const int e = warp + 8 * k;
                kT[e * 32 + lane] = (float)(e & 0xF0) * ((k & 1) ? A1 : A0);
            }
        }
        if (warp == 0) {                                   // C = z0 * sum_j q'_z,j
            float c = sQ[3 * lane];
            #pragma unroll
            for (int off = 16; off >= 1; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
            if (lane == 0) sC[0] = c * z0;
        }
        named_bar_sync(1, nthr);
        // z coefficient per code of this lane: q'_z,j * dz / 256 (the code bits give 256 i_z)
        const int j1 = 2 * l16 + half, j2 = 2 * l16 + 1 - half;
        const float2 az = make_float2(sQ[3 * j1] * dz * (1.f / 256.f), sQ[3 * j2] * dz * (1.f / 256.f));
        const float C = sC[0];

        float mrun = -INFINITY, lsum = 0.f;
        float2 azz[4], axy[8];
        #pragma unroll
        for (int k = 0; k < 4; ++k) azz[k] = make_float2(0.f, 0.f);
        #pragma unroll
        for (int k = 0; k < 8; ++k) axy[k] = make_float2(0.f, 0.f);
        for (int tile = 0; tile < ntiles; ++tile, ++seq) {
            if (tile + 1 == ntiles)                      // the finish and the next rotation read R
                for (int i = tid; i < R_LINES; i += nthr) prefetch_l2(p.R + i * 32);
            const int s = seq % STAGES;
            if (alive && !mbar_wait(&full[s], (seq / STAGES) & 1, kErrWaitFull)) alive = false;
            const int nt = min(TT, ntok - tile * TT);
            if (alive && warp * 32 < nt) {
                const uint8_t* stg = smem + OFF_STAGE + s * STAGE;
                // ---- K: 32 scores of this warp's tokens ------------------------------
                const uint32_t* K32 = reinterpret_cast<const uint32_t*>(stg) + warp * 512;
                float ps[16];
                #pragma unroll
                for (int st = 0; st < 16; ++st) {
                    const uint32_t w = K32[st * 32 + lane];           // token 2 st + half, word l16
                    const uint32_t i1 = __byte_perm(w, 0u, selr1), i2 = __byte_perm(w, 0u, selr2);
                    const float2 zz = fadd2(make_float2(__int_as_float(__byte_perm(w, 0x4B000000u, selz1)),
                                                        __int_as_float(__byte_perm(w, 0x4B000000u, selz2))),
                                            make_float2(-MAGIC, -MAGIC));
                    const float t1 = lds_f32(kb1 + i1 * 128u);
                    const float t2 = lds_f32(kb2 + i2 * 128u);
                    const float2 a = ffma2(az, zz, make_float2(t1, t2));
                    ps[st] = a.x + a.y;
                }
                transpose_reduce16(ps, lane);
                const int tk = warp * 32 + 2 * l16 + half;            // token of ps[0]
                const float sc = (tk < nt) ? ps[0] + C : -INFINITY;
                if (__any_sync(0xffffffffu, sc > mrun)) {             // rare after the first tiles
                    float mt = sc;
                    #pragma unroll
                    for (int off = 16; off >= 1; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
                    const float f = fast_exp2(mrun - mt);             // 0 on the first valid tile
                    lsum *= f;
                    #pragma unroll
                    for (int k = 0; k < 4; ++k) azz[k] = fmul2(azz[k], make_float2(f, f));
                    #pragma unroll
                    for (int k = 0; k < 8; ++k) axy[k] = fmul2(axy[k], make_float2(f, f));
                    mrun = mt;
                }
                const float pk = (mrun == -INFINITY) ? 0.f : fast_exp2(sc - mrun);
                lsum += pk;
                // ---- V: weighted sums of this warp's tokens --------------------------
                const uint4* V16 = reinterpret_cast<const uint4*>(stg + TILE) + warp * 128;
                #pragma unroll
                for (int st = 0; st < 4; ++st) {
                    // token 8 st + tg: its weight sits in lane 16 (tg & 1) + 4 st + tg / 2
                    const float pw = __shfl_sync(0xffffffffu, pk, 16 * (tg & 1) + 4 * st + (tg >> 1));
                    const uint4 wv = V16[st * 32 + lane];
                    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
                    #pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        const uint32_t w = ww[h];
                        // low code (triplet 8 q4 + 2h), high code (8 q4 + 2h + 1)
                        const float2 zf = fadd2(make_float2(__int_as_float((w & 0xF00u) | 0x4B000000u),
                                                            __int_as_float(__byte_perm(w, 0x4B000000u, 0x7534))),
                                                make_float2(-MAGIC, -MAGIC));
                        const float2 rf = fadd2(make_float2(__int_as_float((w & 0xF0u) | 0x4B000000u),
                                                            __int_as_float(((w >> 16) & 0xF0u) | 0x4B000000u)),
                                                make_float2(-MAGIC, -MAGIC));
                        const float2 cs0 = lds_f32x2(csb | ((w << 3) & 0x78u));      // table is 128-byte aligned
                        const float2 cs1 = lds_f32x2(csb | ((w >> 13) & 0x78u));
                        azz[h] = ffma2(make_float2(pw, pw), zf, azz[h]);
                        const float2 wr = fmul2(make_float2(pw, pw), rf);
                        axy[2 * h] = ffma2(make_float2(wr.x, wr.x), cs0, axy[2 * h]);
                        axy[2 * h + 1] = ffma2(make_float2(wr.y, wr.y), cs1, axy[2 * h + 1]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        {                                                  // prefetch the next item's query
            WorkCursor pc = wc;
            ItemRange rn;
            if (tid < 96 && work_next<false>(p, pc, rn))
                qreg = q_load(p.q, p.qdt, (int64_t)rn.b * p.q_bs + (int64_t)rn.hk * p.q_hs + tid);
        }
        // ---- merge: lanes of a warp, then the warps ----------------------------------
        #pragma unroll
        for (int off = 16; off >= 1; off >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
        #pragma unroll
        for (int off = 4; off <= 16; off <<= 1) {
            #pragma unroll
            for (int k = 0; k < 8; ++k) {
                axy[k].x += __shfl_xor_sync(0xffffffffu, axy[k].x, off);
                axy[k].y += __shfl_xor_sync(0xffffffffu, axy[k].y, off);
            }
            #pragma unroll
            for (int k = 0; k < 4; ++k) {
                azz[k].x += __shfl_xor_sync(0xffffffffu, azz[k].x, off);
                azz[k].y += __shfl_xor_sync(0xffffffffu, azz[k].y, off);
            }
        }
        if (tg == 0) {
            float* o = sAcc + warp * 96 + 24 * q4;          // triplets 8 q4 .. 8 q4 + 7
            #pragma unroll
            for (int h = 0; h < 4; ++h) {
                o[6 * h + 0] = azz[h].x;  o[6 * h + 1] = axy[2 * h].x;      o[6 * h + 2] = axy[2 * h].y;
                o[6 * h + 3] = azz[h].y;  o[6 * h + 4] = axy[2 * h + 1].x;  o[6 * h + 5] = axy[2 * h + 1].y;
            }
        }
        if (lane == 0) {
            sWm[warp] = mrun;
            sWl[warp] = lsum;
        }
        named_bar_sync(1, nthr);
        if (tid < 96) {
            float M = -INFINITY;
            #pragma unroll
            for (int w = 0; w < W; ++w) M = fmaxf(M, sWm[w]);
            float v = 0.f, L = 0.f;
            #pragma unroll
            for (int w = 0; w < W; ++w) {
                const float f = (sWm[w] == -INFINITY) ? 0.f : fast_exp2(sWm[w] - M);
                v = fmaf(f, sAcc[w * 96 + tid], v);
                L = fmaf(f, sWl[w], L);
            }
            // z: sum p (z0 + dz i_z) = z0 l + dz/256 * sum p (256 i_z)
            if (tid % 3 == 0) v = fmaf(dz * (1.f / 256.f), v, z0 * L);
            sAcc[tid] = v;
            if (tid == 0) {
                sM[0] = M;
                sL[0] = L;
            }
        }
        named_bar_sync(1, nthr);
        finish_item(p, r, sM, sL, sAcc, sFin, sflag, p.R, 96, tid, nthr, 4);
    }
    xr_finish_call(p, sAcc, sFin, p.R, 96, tid, nthr, 4);
}

}  // namespace pkv
