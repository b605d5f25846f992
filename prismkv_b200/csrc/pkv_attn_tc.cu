// pkv_attn_tc.cu -- decode attention on 5th-generation tensor cores (head_dim 96,
// bf16 / fp16 queries, any codec: uniform polar, learned codebooks, BiasTable,
// Lloyd-Max z; grouped heads up to 16 per KV head).
//
// Per 128-token tile of one (batch, KV head) item:
//   decoder warps   K and V codes (TMA ring) -> rotated-space triplets through the
//                   codec's decode LUTs (dec_z, dec_xy: bias and Lloyd-Max folded in)
//                   -> bf16 tiles Khat, Vhat [128 tokens][96] in the 64-byte-swizzle
//                   K-major layout (three 32-column chunks)
//   MMA thread      S[128 x 16] = Khat . q'^T        (kind::f16, A K-major, B K-major)
//                   O[128 x 16] = Vhat^T . P^T       (A = Vhat read MN-major, M = 96 -> 128)
//                   fp32 accumulators in tensor memory, two buffers each
//   softmax group   (4 warps, one TMEM lane quarter each) S -> online softmax with the
//                   running max per head, P (bf16) -> shared memory; then accumulates
//                   O into registers with the per-tile rescale exp2(m_old - m_new)
// q' = scale log2(e) R q per head (bf16, rows >= group size zero), set once per item.
// The item ends in finish_item (normalise, apply R, or write / merge split partials).
//
// bf16 MMA inputs give errors of order 2^-9 relative per element; the kernel serves
// bf16 / fp16 queries only, whose stated tolerance is 2e-2 (fp32 queries take the
// fp32 kernels).  Every wait is bounded: on expiry the kernel sets the device
// error word, keeps its control flow (so every named barrier is still met), skips
// further tensor work and frees its tensor memory before returning.

namespace pkv {
namespace atc {

constexpr int TT = 128;                    // tokens per tile (MMA M of the scores)
constexpr int D = 96;
constexpr int NG = 16;                     // MMA N: query heads of the group, padded
constexpr int STAGES = 3;                  // code ring (K and V of a tile per stage)
constexpr int SM_WARPS = 4;                // softmax / accumulate group
// decoder warps: 16 when the softmax group's per-head state is small (groups <= 8), else 8
__host__ __device__ constexpr int dec_warps(int gm) { return gm <= 8 ? 16 : 8; }
__host__ __device__ constexpr int threads_for(int gm) { return (2 + SM_WARPS + dec_warps(gm)) * 32; }
constexpr int STAGE = 2 * TT * 64;         // 16 KB: K and V codes, 12-bit in uint16
constexpr int HCHUNK = TT * 64;            // 8 KB: one 32-column chunk of a decoded tile
constexpr int KH = 3 * HCHUNK;             // Khat tile
// Vhat tiles: 3 chunks each, 24 KB apart.  The PV MMA reads 4 chunks (M = 128 rows): chunk 3 of
// buffer b is chunk 0 of buffer b + 1 (or the zeroed tail after the last one), so output rows
// 96..127 are unused garbage and need no zero padding.
constexpr int NVH = 3;                     // Vhat buffers
constexpr int VHS = 3 * HCHUNK;            // stride between Vhat buffers
constexpr int VH_REGION = NVH * VHS + HCHUNK;
constexpr int PCH = NG * 64;               // 1 KB: P chunk of 32 tokens x 16 heads
constexpr int PT = 4 * PCH;
constexpr int QB = 3 * NG * 64;            // q' operand: 3 chunks of 16 rows
constexpr int OFF_STAGE = 0;
constexpr int OFF_KH = OFF_STAGE + STAGES * STAGE;
constexpr int OFF_VH = OFF_KH + 2 * KH;
constexpr int OFF_P = OFF_VH + VH_REGION;
constexpr int OFF_QB = OFF_P + 2 * PT;
// decode tables already rounded to the operand type: z as one 16-bit value, (x, y) as a packed
// pair, so a code costs two loads and no conversion
constexpr int OFF_LUTZ = OFF_QB + QB;                       // dec_z [<= 256] bf16 / f16
constexpr int OFF_LUTXY = OFF_LUTZ + 256 * 2;               // dec_xy [<= 4096] bf16x2 / f16x2
constexpr int LUTXY_BYTES = 4096 * 4;
constexpr int OFF_M = OFF_LUTXY + LUTXY_BYTES;              // sM, sL [NG], alpha [2][NG], red [4][NG], flag
constexpr int OFF_O = OFF_M + (2 * NG + 2 * NG + SM_WARPS * NG) * 4 + 16;   // sO [NG][96] (finish_item)
constexpr int OFF_FIN = OFF_O + NG * D * 4;                 // sFin [NG][96]; raw queries before the finish
constexpr int OFF_BAR = OFF_FIN + NG * D * 4 + 16;
constexpr int NBAR = 2 * STAGES + 2 * 8 + 2 * NVH + 1;
constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
constexpr int SMEM_BYTES = OFF_TMEM + 16 + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory of the tensor-core attention kernel");
constexpr int TMEM_COLS = 64;              // S[2] at 0, 16; O[2] at 32, 48
// D f32, A and B bf16 (or f16: format 0), N = 16, M = 128; PV additionally A MN-major (bit 15)
__host__ __device__ constexpr uint32_t idesc(uint32_t ab_fmt, bool a_mn) {
    return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | ((a_mn ? 1u : 0u) << 15) | ((uint32_t)(NG >> 3) << 17) |
           ((uint32_t)(TT >> 4) << 24);
}

// 64-byte swizzle, K-major: rows 64 B apart, 8-row groups 512 B apart
__device__ __forceinline__ uint64_t desc_k(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(512u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)4u << 61);
}
// 64-byte swizzle, MN-major: 32-element M chunks HCHUNK apart (leading), 8-row K groups 512 B apart (stride)
__device__ __forceinline__ uint64_t desc_mn(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(HCHUNK >> 4) << 16) | ((uint64_t)(512u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)4u << 61);
}

// byte offset of element (row, col) of a [rows][32k] bf16 tile in 64-byte-swizzle chunks
__device__ __forceinline__ uint32_t sw_off(int row, int col, int chunk_bytes) {
    const int chunk = col >> 5, e = col & 31;
    return (uint32_t)(chunk * chunk_bytes + row * 64 + ((((e >> 3) ^ (row >> 1)) & 3) << 4) + (e & 7) * 2);
}

__device__ __forceinline__ void mma(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.u32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(dtmem), "l"(adesc), "l"(bdesc), "r"(id), "r"(acc) : "memory");
}

__device__ __forceinline__ uint32_t pack2(float a, float b, bool f16) {
    uint32_t r;
    if (f16) asm("cvt.rn.f16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(a), "f"(b));
    else asm("cvt.rn.bf16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(a), "f"(b));
    return r;
}

__device__ __forceinline__ uint16_t half1(float a, bool f16) {
    return (uint16_t)(pack2(a, 0.f, f16) & 0xFFFFu);
}

// N consecutive fp32 columns (N = 4, 8, 16) of this thread's TMEM lane
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float* v) {
    if constexpr (N == 16) {
        etc::tmem_ld16(taddr, *reinterpret_cast<float(*)[16]>(v));
    } else if constexpr (N == 8) {
        etc::tmem_ld8(taddr, v);
    } else {
        uint32_t r[4];
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(taddr));
        #pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
    }
}

}  // namespace atc

// GM: register state per query head of the group (4, 8 or 16 >= the group size)
template <int CB, int GM>
__global__ void __launch_bounds__(atc::threads_for(GM), 1) attn_tc_kernel(AttnParams p) {
    using namespace atc;
    constexpr int DEC_WARPS = dec_warps(GM);
    constexpr int THREADS = threads_for(GM);
    extern __shared__ uint8_t atc_smem_raw[];
    // 1024-byte aligned base for the swizzled operands, derived from the array itself (pointer plus
    // offset) so that every access below stays a shared-memory access
    uint8_t* smem = atc_smem_raw + ((1024u - (smem_u32(atc_smem_raw) & 1023u)) & 1023u);
    const uint32_t sb = smem_u32(smem);
    uint16_t* lutz = reinterpret_cast<uint16_t*>(smem + OFF_LUTZ);
    uint32_t* lutxy = reinterpret_cast<uint32_t*>(smem + OFF_LUTXY);
    float* sM = reinterpret_cast<float*>(smem + OFF_M);
    float* sL = sM + NG;
    float* sAlpha = sL + NG;                 // [2][NG]
    float* sRed = sAlpha + 2 * NG;           // [SM_WARPS][NG]
    int* sflag = reinterpret_cast<int*>(sRed + SM_WARPS * NG);
    float* sO = reinterpret_cast<float*>(smem + OFF_O);
    float* sFin = reinterpret_cast<float*>(smem + OFF_FIN);
    float* sQs = sFin;                       // raw queries of an item, consumed before its finish
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* full = bar;                    // [STAGES] codes landed
    uint64_t* empty = full + STAGES;         // [STAGES] codes consumed (decoder warps)
    uint64_t* kh_full = empty + STAGES;      // [2]
    uint64_t* kh_empty = kh_full + 2;        // [2] scores MMA done with Khat
    uint64_t* vh_full = kh_empty + 2;        // [NVH]
    uint64_t* vh_empty = vh_full + NVH;      // [NVH] PV MMA done with Vhat
    uint64_t* s_full = vh_empty + NVH;       // [2] scores in TMEM
    uint64_t* s_empty = s_full + 2;          // [2] softmax read them
    uint64_t* p_full = s_empty + 2;          // [2] P in shared memory
    uint64_t* p_empty = p_full + 2;          // [2] PV MMA done with P
    uint64_t* o_full = p_empty + 2;          // [2] O tile in TMEM
    uint64_t* o_empty = o_full + 2;          // [2] accumulated
    uint64_t* q_ready = o_empty + 2;         // q' of the next item in place
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // R (36 KB) is read from global memory by the query rotation and the finish; once the code
    // stream runs, a miss on it waits behind the bulk copies, so bring it into L2 first
    constexpr int R_LINES = D * D * 4 / 128;
    for (int i = tid; i < R_LINES; i += THREADS) prefetch_l2(p.R + i * 32);
    const bool f16 = (p.qdt == PKV_F16);
    const uint32_t ab = f16 ? 0u : 1u;
    const int bf = p.bits_flat;
    const uint32_t cmask = (uint32_t)p.code_mask, fmask = (uint32_t)p.flat_mask;

    // ---- set-up: LUTs, zero padding of the operands, barriers, tensor memory ----
    for (int i = tid; i < p.Cz; i += THREADS) lutz[i] = half1(__ldg(p.dec_z + i), f16);
    for (int i = tid; i < p.n_xy; i += THREADS) {
        const float2 xy = __ldg(reinterpret_cast<const float2*>(p.dec_xy) + i);
        lutxy[i] = pack2(xy.x, xy.y, f16);
    }
    for (int i = tid; i < VH_REGION / 16; i += THREADS)           // Vhat tiles and the tail: finite
        reinterpret_cast<uint4*>(smem + OFF_VH)[i] = make_uint4(0, 0, 0, 0);
    for (int i = tid; i < (2 * PT + QB) / 16; i += THREADS)
        reinterpret_cast<uint4*>(smem + OFF_P)[i] = make_uint4(0, 0, 0, 0);
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], DEC_WARPS);
        }
        for (int b = 0; b < NVH; ++b) {
            mbar_init(&vh_full[b], DEC_WARPS);
            mbar_init(&vh_empty[b], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&kh_full[b], DEC_WARPS);
            mbar_init(&kh_empty[b], 1);
            mbar_init(&s_full[b], 1);
            mbar_init(&s_empty[b], SM_WARPS);
            mbar_init(&p_full[b], SM_WARPS);
            mbar_init(&p_empty[b], 1);
            mbar_init(&o_full[b], 1);
            mbar_init(&o_empty[b], SM_WARPS);
        }
        mbar_init(q_ready, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_proxy_async_smem();
    etc::tc_fence_before();
    __syncthreads();
    etc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer: K and V codes of every tile ----------------
        if (lane == 0) produce<TT, true, false>(p, smem + OFF_STAGE, STAGE, full, empty, DEC_WARPS, CB);
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t id_s = idesc(ab, false), id_o = idesc(ab, true);
            bool alive = true;
            int it = 0, items = 0;
            WorkCursor wc = work_begin(p);
            ItemRange r;
            auto scores = [&](int t) {
                const int b = t & 1;
                if (alive && !mbar_wait_spin(&kh_full[b], (t >> 1) & 1, kErrWaitFull)) alive = false;
                if (alive && t >= 2 && !mbar_wait_spin(&s_empty[b], ((t >> 1) - 1) & 1, kErrWaitEmpty)) alive = false;
                if (!alive) return;
                etc::tc_fence_after();
                #pragma unroll
                for (int k = 0; k < D / 16; ++k)
                    mma(tmem + (uint32_t)(b * NG), desc_k(sb + OFF_KH + b * KH + (k >> 1) * HCHUNK + (k & 1) * 32),
                        desc_k(sb + OFF_QB + (k >> 1) * (NG * 64) + (k & 1) * 32), id_s, k != 0);
                etc::mma_commit(smem_u32(&kh_empty[b]));
                etc::mma_commit(smem_u32(&s_full[b]));
            };
            auto pv = [&](int t) {
                const int b = t & 1, b3 = t % NVH;
                if (alive && !mbar_wait_spin(&p_full[b], (t >> 1) & 1, kErrWaitFull)) alive = false;
                if (alive && !mbar_wait_spin(&vh_full[b3], (t / NVH) & 1, kErrWaitFull)) alive = false;
                if (alive && t >= 2 && !mbar_wait_spin(&o_empty[b], ((t >> 1) - 1) & 1, kErrWaitEmpty)) alive = false;
                if (!alive) return;
                etc::tc_fence_after();
                #pragma unroll
                for (int k = 0; k < TT / 16; ++k)
                    mma(tmem + (uint32_t)(32 + b * NG), desc_mn(sb + OFF_VH + b3 * VHS + k * 1024),
                        desc_k(sb + OFF_P + b * PT + (k >> 1) * PCH + (k & 1) * 32), id_o, k != 0);
                etc::mma_commit(smem_u32(&vh_empty[b3]));
                etc::mma_commit(smem_u32(&p_empty[b]));
                etc::mma_commit(smem_u32(&o_full[b]));
            };
            while (work_next<false>(p, wc, r)) {
                const int nt = (r.tok1 - r.tok0 + TT - 1) / TT;
                if (nt == 0) continue;
                if (alive && !mbar_wait_spin(q_ready, items & 1, kErrWaitFull)) alive = false;
                ++items;
                scores(it);
                for (int j = 0; j < nt; ++j) {
                    if (j + 1 < nt) scores(it + j + 1);      // keep the next tile's scores ahead of PV
                    pv(it + j);
                }
                it += nt;
            }
            // the last MMAs must be complete before tensor memory is freed
            if (it > 0) mbar_wait_spin(&o_full[(it - 1) & 1], ((it - 1) >> 1) & 1, kErrWaitDrain);
        }
    } else if (warp >= 2 + SM_WARPS) {
        // ---------------- decoders: codes -> bf16 Khat / Vhat ----------------
        const int dt = tid - (2 + SM_WARPS) * 32;              // 0..255
        bool alive = true;
        int it = 0, seq = 0;
        WorkCursor wc = work_begin(p);
        ItemRange r;
        while (work_next<false>(p, wc, r)) {
            const int nt = (r.tok1 - r.tok0 + TT - 1) / TT;
            for (int j = 0; j < nt; ++j, ++it, ++seq) {
                const int s = seq % STAGES, b = it & 1, b3 = it % NVH;
                if (alive && !mbar_wait_spin(&full[s], (seq / STAGES) & 1, kErrWaitFull)) alive = false;
                // thread -> (token t0 + i * TSTEP, triplet pair jp); the swizzle key (t >> 1) & 3 is the
                // same for all its tokens (TSTEP is a multiple of 8), so the three store offsets are
                // fixed and advance by TSTEP rows per step
                constexpr int NTH = DEC_WARPS * 32, TSTEP = NTH / 16;
                const int jp = dt & 15, t0 = dt >> 4;
                const uint32_t o0 = sw_off(t0, 6 * jp, HCHUNK), o1 = sw_off(t0, 6 * jp + 2, HCHUNK),
                               o2 = sw_off(t0, 6 * jp + 4, HCHUNK);
                const uint8_t* stage = smem + OFF_STAGE + s * STAGE;
                // K first (its buffer frees as soon as the scores MMA is done), then V (its buffer
                // frees only after the PV MMA of the tile NVH back)
                #pragma unroll 1
                for (int kv = 0; kv < 2; ++kv) {
                    if (kv == 0) {
                        if (alive && it >= 2 && !mbar_wait_spin(&kh_empty[b], ((it >> 1) - 1) & 1, kErrWaitEmpty))
                            alive = false;
                    } else {
                        if (alive && it >= NVH && !mbar_wait_spin(&vh_empty[b3], ((it / NVH) - 1) & 1, kErrWaitEmpty))
                            alive = false;
                    }
                    if (alive) {
                        const uint8_t* codes = stage + kv * TT * 32 * CB + t0 * 32 * CB + jp * 2 * CB;
                        uint8_t* dst = smem + (kv == 0 ? OFF_KH + b * KH : OFF_VH + b3 * VHS);
                        #pragma unroll
                        for (int i = 0; i < TT / TSTEP; ++i) {
                            uint32_t c0, c1;
                            if (CB == 2) {
                                const uint32_t word = *reinterpret_cast<const uint32_t*>(codes + i * TSTEP * 64);
                                c0 = word & 0xFFFFu;
                                c1 = word >> 16;
                            } else {
                                const uint32_t half = *reinterpret_cast<const uint16_t*>(codes + i * TSTEP * 32);
                                c0 = half & 0xFFu;
                                c1 = half >> 8;
                            }
                            c0 &= cmask;
                            c1 &= cmask;
                            const uint32_t z0 = lutz[c0 >> bf], z1 = lutz[c1 >> bf];
                            const uint32_t xy0 = lutxy[p.xy_per_z ? c0 : (c0 & fmask)];
                            const uint32_t xy1 = lutxy[p.xy_per_z ? c1 : (c1 & fmask)];
                            uint8_t* d = dst + i * TSTEP * 64;
                            // dims 6jp .. 6jp+5 = z0 x0 | y0 z1 | x1 y1
                            *reinterpret_cast<uint32_t*>(d + o0) = __byte_perm(z0, xy0, 0x5410);
                            *reinterpret_cast<uint32_t*>(d + o1) = __byte_perm(xy0, z1, 0x5432);
                            *reinterpret_cast<uint32_t*>(d + o2) = xy1;
                        }
                        fence_proxy_async_smem();             // generic stores -> tensor-core reads
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(kv == 0 ? &kh_full[b] : &vh_full[b3]);
                }
                if (lane == 0) mbar_arrive(&empty[s]);
            }
        }
    } else {
        // ---------------- softmax / accumulate group (warps 2..5) ----------------
        const int gt = tid - 64;                 // 0..127
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;     // TMEM lane: a token (S) or a dimension (O)
        const int G = p.G;
        const int nthr = SM_WARPS * 32;
        bool alive = true;
        int it = 0, items = 0;
        WorkCursor wc = work_begin(p);
        ItemRange r;
        while (work_next<false>(p, wc, r)) {
            const int ntok = r.tok1 - r.tok0;
            const int nt = (ntok + TT - 1) / TT;
            float m_run[GM], l_run[GM], acc[GM];
            #pragma unroll
            for (int g = 0; g < GM; ++g) { m_run[g] = -INFINITY; l_run[g] = 0.f; acc[g] = 0.f; }
            if (nt > 0) {
                // q' = scale log2(e) R q for the group's heads -> bf16 operand rows (rows >= G stay zero)
                for (int idx = gt; idx < G * D; idx += nthr) {
                    const int g = idx / D, i = idx % D;
                    sQs[idx] = q_load(p.q, p.qdt, (int64_t)r.b * p.q_bs + (int64_t)(r.hk * G + g) * p.q_hs + i);
                }
                named_bar_sync(1, nthr);
                // one warp per row k of R, lanes over the input index: each row is three coalesced
                // 128-byte loads from L2, shared by the group's heads; six rows' loads are in
                // flight at once, so the 24 rows of a warp cost four memory round trips
                constexpr int RB = 6, ROWS = D / SM_WARPS;
                static_assert(ROWS % RB == 0, "rows per batch");
                for (int k0 = 0; k0 < ROWS; k0 += RB) {
                    float rv[RB][3];
                    #pragma unroll
                    for (int u = 0; u < RB; ++u) {
                        const float* Rk = p.R + (quarter + SM_WARPS * (k0 + u)) * D;
                        rv[u][0] = __ldg(Rk + lane);
                        rv[u][1] = __ldg(Rk + lane + 32);
                        rv[u][2] = __ldg(Rk + lane + 64);
                    }
                    for (int g = 0; g < G; ++g) {
                        const float* qg = sQs + g * D;
                        const float qa = qg[lane], qb = qg[lane + 32], qc = qg[lane + 64];
                        #pragma unroll
                        for (int u = 0; u < RB; ++u) {
                            float v = fmaf(rv[u][0], qa, fmaf(rv[u][1], qb, rv[u][2] * qc));
                            #pragma unroll
                            for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                            if (lane == 0)
                                *reinterpret_cast<uint16_t*>(smem + OFF_QB +
                                                             sw_off(g, quarter + SM_WARPS * (k0 + u), NG * 64)) =
                                    half1(v * p.scale_log2, f16);
                        }
                    }
                }
                fence_proxy_async_smem();
                named_bar_sync(1, nthr);
                if (gt == 0) mbar_arrive(q_ready);
                ++items;
            }
            for (int j = 0; j <= nt; ++j) {
                if (j + 1 == nt)                         // the finish reads R: back into L2
                    for (int i = gt; i < R_LINES; i += nthr) prefetch_l2(p.R + i * 32);
                // ---- softmax of tile j ----
                if (j < nt) {
                    const int t = it + j, b = t & 1;
                    bool ok = alive && mbar_wait_spin(&s_full[b], (t >> 1) & 1, kErrWaitFull);
                    if (ok && t >= 2) ok = mbar_wait_spin(&p_empty[b], ((t >> 1) - 1) & 1, kErrWaitEmpty);
                    alive = __all_sync(0xffffffffu, ok) && alive;
                    float sv[GM];
                    if (alive) {
                        etc::tc_fence_after();
                        tmem_ld<GM>(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * NG), sv);
                        etc::tmem_wait_ld();
                        etc::tc_fence_before();
                    } else {
                        #pragma unroll
                        for (int g = 0; g < GM; ++g) sv[g] = 0.f;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s_empty[b]);
                    const bool valid = (j * TT + row) < ntok;
                    // tile max per head over the 128 tokens
                    #pragma unroll
                    for (int g = 0; g < GM; ++g) {
                        float v = (valid && g < G) ? sv[g] : -INFINITY;
                        #pragma unroll
                        for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
                        if (lane == 0) sRed[quarter * NG + g] = v;
                    }
                    named_bar_sync(1, nthr);
                    uint8_t* P = smem + OFF_P + b * PT;
                    #pragma unroll
                    for (int g = 0; g < GM; ++g) {
                        if (g >= G) break;
                        float tm = sRed[g];
                        #pragma unroll
                        for (int q = 1; q < SM_WARPS; ++q) tm = fmaxf(tm, sRed[q * NG + g]);
                        const float mn = fmaxf(m_run[g], tm);
                        const float alpha = (m_run[g] == -INFINITY) ? 0.f : fast_exp2(m_run[g] - mn);
                        m_run[g] = mn;
                        const float pv = valid ? fast_exp2(sv[g] - mn) : 0.f;
                        l_run[g] = fmaf(l_run[g], alpha, pv);
                        if (gt == 0) sAlpha[b * NG + g] = alpha;
                        *reinterpret_cast<uint16_t*>(P + sw_off(g, row, PCH)) = half1(pv, f16);
                    }
                    fence_proxy_async_smem();
                    named_bar_sync(1, nthr);                 // sRed reads done; alpha and P written
                    if (lane == 0) mbar_arrive(&p_full[b]);
                }
                // ---- accumulate tile j - 1 ----
                if (j >= 1) {
                    const int t = it + j - 1, b = t & 1;
                    bool ok = alive && mbar_wait_spin(&o_full[b], (t >> 1) & 1, kErrWaitFull);
                    alive = __all_sync(0xffffffffu, ok) && alive;
                    float ov[GM];
                    if (alive) {
                        etc::tc_fence_after();
                        tmem_ld<GM>(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(32 + b * NG), ov);
                        etc::tmem_wait_ld();
                        etc::tc_fence_before();
                    } else {
                        #pragma unroll
                        for (int g = 0; g < GM; ++g) ov[g] = 0.f;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&o_empty[b]);
                    #pragma unroll
                    for (int g = 0; g < GM; ++g) acc[g] = fmaf(acc[g], sAlpha[b * NG + g], ov[g]);
                    // sAlpha[b] is rewritten by the softmax of tile t + 2, which follows this read
                }
            }
            it += nt;
            // ---- finish: M (log2 units), l, unnormalised rotated output per head ----
            #pragma unroll
            for (int g = 0; g < GM; ++g) {
                float l = l_run[g];
                #pragma unroll
                for (int off = 16; off >= 1; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
                if (lane == 0) sRed[quarter * NG + g] = l;
            }
            if (row < D) {
                #pragma unroll
                for (int g = 0; g < GM; ++g)
                    if (g < G) sO[g * D + row] = acc[g];
            }
            named_bar_sync(1, nthr);
            #pragma unroll
            for (int g = 0; g < GM; ++g) {
                if (gt == g && g < G) {
                    float l = 0.f;
                    for (int q = 0; q < SM_WARPS; ++q) l += sRed[q * NG + g];
                    sL[g] = l;
                    sM[g] = m_run[g];
                }
            }
            named_bar_sync(1, nthr);
            finish_item(p, r, sM, sL, sO, sFin, sflag, p.R, D, gt, nthr, 1);
        }
        xr_finish_call(p, sO, sFin, p.R, D, gt, nthr, 1);
    }
    etc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        etc::tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

}  // namespace pkv
