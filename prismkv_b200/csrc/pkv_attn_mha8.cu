// pkv_attn_mha8.cu -- decode attention over one-byte codes: head_dim 96, uniform-polar
// (x, y) cells (at most 32 (r, theta) cells), uniform z bins, no BiasTable; one query
// head per work unit (MHA, or grouped heads with every query head its own unit).
//
// One CTA per SM, one pass over an item's tokens.  The K and V codes of a 512-token tile
// arrive together in one ring stage; each of the 16 consumer warps owns 32 tokens of every
// tile and keeps its own running max, sum of weights and V accumulators (online softmax per
// warp, rescaled only when a warp vote sees a score above the running max); the warps'
// states merge once per item, then finish_item normalises and applies R (resident in
// shared memory for the CTA's lifetime).
//
//  * K: score table T[c][j] = q'_j . (z, x, y)(c) over all 256 byte values c and the 32
//    triplets j (32 KB), z and (x, y) straight from the codec's decode tables.  Lane l
//    reads word l%8 of token 4s + l/8 (four codes) and takes the word's bytes starting at
//    byte l/8, so the 32 table loads of a step hit 32 distinct banks.
//    An 8-lane transpose-reduce completes 32 scores per 8 steps.
//  * V: lane l reads 8 codes (triplets 8(l%4)..+7) of token l/4 of a group of 8 tokens.
//    Each byte is moved to bits 8..15 of a word.  z comes from its bits under the 2^23
//    float exponent (uniform bins are affine in i_z); (x, y) from the (r, theta) cell
//    table, whose rows sit 256 bytes apart on an 8 KB boundary, so one AND-OR of the
//    word with the lane's table address gives the load address.  Each row holds 16 copies
//    of its (x, y) and lane l reads copy l%16: a half-warp's 8-byte loads hit 32 banks.
//
// Every mbarrier wait is bounded (device error word on expiry, control flow kept).

namespace pkv {
namespace mha8 {
constexpr int W = 16;                                  // consumer warps (one CTA per SM)
constexpr int TT = 32 * W;                             // tokens per tile (32 per warp)
constexpr int STAGES = 4;
constexpr int ROW = 32;                                // 32 one-byte codes per token
constexpr int TILE = TT * ROW;                         // K (or V) codes of a tile
constexpr int STAGE = 2 * TILE;                        // K then V
constexpr int XY_ALIGN = 8192;                         // (r, theta) table: 32 rows x 256 bytes
constexpr int OFF_XY = 0;
constexpr int OFF_STAGE = OFF_XY + XY_ALIGN;
constexpr int RBYTES = 96 * 96 * 4;                    // R, fp32, row pitch 96, resident
constexpr int OFF_R = OFF_STAGE + STAGES * STAGE;
constexpr int OFF_KT = OFF_R + RBYTES;                 // [256][32] score table
constexpr int OFF_Z = OFF_KT + 256 * 32 * 4;           // dec_z [<= 256]
constexpr int OFF_Q = OFF_Z + 256 * 4;                 // [96] rotated query
constexpr int OFF_QRAW = OFF_Q + 96 * 4;               // [96] raw query
constexpr int OFF_ACC = OFF_QRAW + 96 * 4;             // [W][96] per-warp accumulators
constexpr int OFF_FIN = OFF_ACC + W * 96 * 4;          // [96]
constexpr int OFF_WML = OFF_FIN + 96 * 4;              // [W] max, [W] sum
constexpr int OFF_MISC = OFF_WML + 2 * W * 4;          // sM, sL, flag
constexpr int OFF_BAR = OFF_MISC + 16;                 // full[STAGES], empty[STAGES], rbar
constexpr int LAYOUT = OFF_BAR + (2 * STAGES + 1) * 8;
constexpr int TOTAL = LAYOUT + XY_ALIGN;               // slack to put the layout on an 8 KB boundary
constexpr float MAGIC = 8388608.f;                     // 2^23
static_assert(OFF_STAGE % 128 == 0 && OFF_R % 128 == 0 && OFF_KT % 128 == 0 && OFF_BAR % 8 == 0, "alignment");
static_assert(TOTAL <= 227 * 1024, "shared memory of the one-byte attention kernel");
}  // namespace mha8

// 8-lane transpose-reduce within each group of 8 lanes: on exit v[0] of lane l holds the
// sum over the 8 lanes of its group of their v[l % 8].
__device__ __forceinline__ void transpose_reduce8(float (&v)[8], int lane) {
    #pragma unroll
    for (int off = 4; off >= 1; off >>= 1) {
        const bool upper = (lane & off) != 0;
        #pragma unroll
        for (int i = 0; i < off; ++i) {
            float send = upper ? v[i] : v[i + off];
            float keep = upper ? v[i + off] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
}

__global__ void __launch_bounds__(mha8::W * 32 + 32, 1) attn_mha8_kernel(AttnParams p) {
    using namespace mha8;
    extern __shared__ __align__(128) uint8_t mha8_smem[];
    // the (r, theta) table's row bits must be free in its base address: put the layout on 8 KB
    uint8_t* smem = mha8_smem + ((XY_ALIGN - ((uint32_t)__cvta_generic_to_shared(mha8_smem) & (XY_ALIGN - 1))) &
                                 (XY_ALIGN - 1));
    float* kT = reinterpret_cast<float*>(smem + OFF_KT);       // score table
    float* sR = reinterpret_cast<float*>(smem + OFF_R);        // R, loaded once
    float* sXY = reinterpret_cast<float*>(smem + OFF_XY);
    float* sZ = reinterpret_cast<float*>(smem + OFF_Z);
    float* sQ = reinterpret_cast<float*>(smem + OFF_Q);
    float* sQraw = reinterpret_cast<float*>(smem + OFF_QRAW);
    float* sAcc = reinterpret_cast<float*>(smem + OFF_ACC);
    float* sFin = reinterpret_cast<float*>(smem + OFF_FIN);
    float* sWm = reinterpret_cast<float*>(smem + OFF_WML);
    float* sWl = sWm + W;
    float* sM = reinterpret_cast<float*>(smem + OFF_MISC);
    float* sL = sM + 1;
    int* sflag = reinterpret_cast<int*>(sM + 2);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* empty = full + STAGES;
    uint64_t* rbar = empty + STAGES;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bf = p.bits_flat;
    const int n_xy = 1 << bf, cz = 1 << p.bits_z;
    const float z0 = __ldg(p.dec_z), dz = __ldg(p.dec_z + 1) - z0;     // uniform z bins: z = z0 + i dz

    for (int i = tid; i < n_xy * 16; i += blockDim.x) {                 // 16 copies of every cell's (x, y)
        const int fl = i >> 4, c = i & 15;
        sXY[fl * 64 + 2 * c] = __ldg(p.dec_xy + 2 * fl);
        sXY[fl * 64 + 2 * c + 1] = __ldg(p.dec_xy + 2 * fl + 1);
    }
    for (int i = tid; i < cz; i += blockDim.x) sZ[i] = __ldg(p.dec_z + i);
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        mbar_init(rbar, 1);
        fence_mbar_init();
        // R, ahead of the code stream; it stays for every item's rotation and finish
        mbar_arrive_expect_tx(rbar, RBYTES);
        bulk_g2s(sR, p.R, RBYTES, rbar);
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
        if (lane == 0) produce<TT, true, false>(p, smem + OFF_STAGE, STAGE, full, empty, W, 1);
        return;
    }

    constexpr int nthr = W * 32;
    // K: lane = (token-in-4 g, word i); byte b_k = (k + g) & 3 of the word at step k
    const int kg = lane >> 3, ki = lane & 7;
    uint32_t ksel[4], kcol[4];
    #pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t b = (uint32_t)((k + kg) & 3);
        ksel[k] = 0x4440u | b;                              // byte b to byte 0, zeros above
        kcol[k] = (uint32_t)__cvta_generic_to_shared(kT) + 4u * (4u * ki + b);
    }
    // V: lane = (token-in-8 tg, 8-triplet chunk q4)
    const int tg = lane >> 2, q4 = lane & 3;
    const uint32_t xyl = (uint32_t)__cvta_generic_to_shared(sXY) + 8u * (lane & 15);
    const uint32_t fm = (uint32_t)(n_xy - 1) << 8;                      // flat cell bits at 8..
    const uint32_t zm = (uint32_t)(cz - 1) << (8 + bf);                 // z bits above them
    const float dzs = dz * exp2f((float)-(8 + bf));                     // per unit of the z field
    int seq = 0;
    bool alive = true;
    if (!mbar_wait(rbar, 0, kErrWaitFull)) alive = false;               // R in place
    WorkCursor wc = work_begin(p);
    ItemRange r;
    while (work_next<false>(p, wc, r)) {
        const int ntok = r.tok1 - r.tok0;
        const int ntiles = (ntok + TT - 1) / TT;
        if (tid < 96) sQraw[tid] = qreg;
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
        // score table: row c (byte value), column j (triplet); warp w fills rows w + W k,
        // lane j column j.  The previous item's last table reads are behind the barrier above.
        {
            const float qz = sQ[3 * lane], qx = sQ[3 * lane + 1], qy = sQ[3 * lane + 2];
            #pragma unroll 4
            for (int k = 0; k < 256 / W; ++k) {
                const int c = (warp + W * k) & p.code_mask;
                const int fl = c & (n_xy - 1);
                kT[(warp + W * k) * 32 + lane] = fmaf(qz, sZ[c >> bf], fmaf(qx, sXY[fl * 64], qy * sXY[fl * 64 + 1]));
            }
        }
        named_bar_sync(1, nthr);

        float mrun = -INFINITY, lsum = 0.f;
        float2 az[4], axy[8];
        #pragma unroll
        for (int k = 0; k < 4; ++k) az[k] = make_float2(0.f, 0.f);
        #pragma unroll
        for (int k = 0; k < 8; ++k) axy[k] = make_float2(0.f, 0.f);
        for (int tile = 0; tile < ntiles; ++tile, ++seq) {
            const int s = seq % STAGES;
            if (alive && !mbar_wait(&full[s], (seq / STAGES) & 1, kErrWaitFull)) alive = false;
            const int nt = min(TT, ntok - tile * TT);
            if (alive && warp * 32 < nt) {
                const uint8_t* stg = smem + OFF_STAGE + s * STAGE;
                // ---- K: 32 scores of this warp's tokens ------------------------------
                const uint32_t* K32 = reinterpret_cast<const uint32_t*>(stg) + warp * 256;
                float ps[8];
                #pragma unroll
                for (int st = 0; st < 8; ++st) {
                    const uint32_t w = K32[st * 32 + lane];           // word ki of token 4 st + kg
                    float t[4];
                    #pragma unroll
                    for (int k = 0; k < 4; ++k) t[k] = lds_f32(kcol[k] + (__byte_perm(w, 0u, ksel[k]) << 7));
                    ps[st] = (t[0] + t[1]) + (t[2] + t[3]);
                }
                transpose_reduce8(ps, lane);
                const int tokk = warp * 32 + 4 * ki + kg;             // token of ps[0]
                const float sc = (tokk < nt) ? ps[0] : -INFINITY;
                if (__any_sync(0xffffffffu, sc > mrun)) {             // rare after the first tiles
                    float mt = sc;
                    #pragma unroll
                    for (int off = 16; off >= 1; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
                    const float f = fast_exp2(mrun - mt);             // 0 on the first valid tile
                    lsum *= f;
                    #pragma unroll
                    for (int k = 0; k < 4; ++k) az[k] = fmul2(az[k], make_float2(f, f));
                    #pragma unroll
                    for (int k = 0; k < 8; ++k) axy[k] = fmul2(axy[k], make_float2(f, f));
                    mrun = mt;
                }
                const float pk = (mrun == -INFINITY) ? 0.f : fast_exp2(sc - mrun);
                lsum += pk;
                // ---- V: weighted sums of this warp's tokens --------------------------
                const uint2* V64 = reinterpret_cast<const uint2*>(stg + TILE) + warp * 128;
                #pragma unroll
                for (int st = 0; st < 4; ++st) {
                    // token 8 st + tg: its weight sits in lane 8 ((8 st + tg) % 4) + (8 st + tg) / 4
                    const float pw = __shfl_sync(0xffffffffu, pk, 8 * (tg & 3) + 2 * st + (tg >> 2));
                    const uint2 wv = V64[st * 32 + lane];
                    const float2 pp = make_float2(pw, pw);
                    #pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t w = h ? wv.y : wv.x;
                        const uint32_t u[4] = {w << 8, w, w >> 8, w >> 16};     // byte k at bits 8..15
                        #pragma unroll
                        for (int k = 0; k < 4; k += 2) {
                            const float2 zf = fadd2(make_float2(__int_as_float((u[k] & zm) | 0x4B000000u),
                                                                __int_as_float((u[k + 1] & zm) | 0x4B000000u)),
                                                    make_float2(-MAGIC, -MAGIC));
                            az[2 * h + k / 2] = ffma2(pp, zf, az[2 * h + k / 2]);
                        }
                        #pragma unroll
                        for (int k = 0; k < 4; ++k)
                            axy[4 * h + k] = ffma2(pp, lds_f32x2((u[k] & fm) | xyl), axy[4 * h + k]);
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
                az[k].x += __shfl_xor_sync(0xffffffffu, az[k].x, off);
                az[k].y += __shfl_xor_sync(0xffffffffu, az[k].y, off);
            }
        }
        if (tg == 0) {
            float* o = sAcc + warp * 96 + 24 * q4;          // triplets 8 q4 .. 8 q4 + 7
            #pragma unroll
            for (int k = 0; k < 4; ++k) {
                o[6 * k + 0] = az[k].x;  o[6 * k + 1] = axy[2 * k].x;      o[6 * k + 2] = axy[2 * k].y;
                o[6 * k + 3] = az[k].y;  o[6 * k + 4] = axy[2 * k + 1].x;  o[6 * k + 5] = axy[2 * k + 1].y;
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
            // z: sum p (z0 + dz i_z) = z0 l + dz 2^-(8+bf) sum p (i_z 2^(8+bf))
            if (tid % 3 == 0) v = fmaf(dzs, v, z0 * L);
            sAcc[tid] = v;
            if (tid == 0) {
                sM[0] = M;
                sL[0] = L;
            }
        }
        named_bar_sync(1, nthr);
        finish_item(p, r, sM, sL, sAcc, sFin, sflag, sR, 96, tid, nthr, 4);
    }
    xr_finish_call(p, sAcc, sFin, sR, 96, tid, nthr, 4);
    // a copy of R that never landed must not outlive the CTA
    if (tid == 0 && !alive) mbar_wait(rbar, 0, kErrWaitDrain);
}

}  // namespace pkv
