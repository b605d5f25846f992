// pkv_encode_tc.cu -- encode with the rotation on 5th-generation tensor cores.
//
// rot = x @ R^T for head_dim 96 and bf16 inputs runs as tcgen05.mma
// (kind::f16, BF16 operands, FP32 accumulator in tensor memory):
//   D[128 vectors x 96] = X[128 x 96] . (R1 + R2 + R3)^T
// with R split on the host into three bf16 parts (R1 = bf16(R),
// R2 = bf16(R - R1), R3 = bf16(R - R1 - R2); the residual is below 2^-26 |R|).
// bf16 x bf16 products are exact, so the accumulator holds the fp32 rotation
// up to summation rounding -- the same class of error as the reference's fp32
// GEMM, which is what the encode parity (bit-exact codes except rounding ties)
// is stated against.  The binning epilogue is encode_triplet, shared with the
// CUDA-core kernel.
//
// One CTA per SM, persistent over 128-vector tiles, warp-specialised:
//   warp 0     TMA producer: X tiles (3 boxes of 32 bf16 columns, 64-byte
//              swizzle) into a 4-stage ring; the R parts once.
//   warp 1     owns the tensor memory (256 columns = two accumulators) and
//              one lane issues the 18 MMAs of a tile (3 parts x 6 K-steps).
//   warps 2-17 epilogue: each TMEM lane quarter is read by four warps, one per
//              quarter of the 32 triplets; tcgen05.ld -> bins -> 8 packed codes
//              per thread, written with one vector store.
// Every mbarrier wait is bounded; on expiry the kernel sets the device error
// word, drains what it issued and frees its tensor memory before returning.

#include <cuda.h>

namespace pkv {
namespace etc {

constexpr int BM = 128;                    // vectors per tile = MMA M
constexpr int D = 96;                      // head dim = MMA N = K
constexpr int STAGES = 4;
constexpr int NPART = 3;                   // bf16 parts of R
constexpr int CHUNK_K = 32;                // bf16 columns per 64-byte swizzle atom
constexpr int A_CHUNK = BM * 64;           // 8 KB: one 32-column slice of a tile
constexpr int A_TILE = 3 * A_CHUNK;        // 24 KB
constexpr int B_CHUNK = D * 64;            // 6 KB
constexpr int B_PART = 3 * B_CHUNK;        // 18 KB
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * A_TILE;
constexpr int OFF_THR = OFF_B + NPART * B_PART;
constexpr int THR_FLOATS = 3 * 255;
constexpr int OFF_CB = OFF_THR + THR_FLOATS * 4 + 4;        // learned codebook copy (16-byte aligned below)
constexpr int CB_BYTES = 32 * 1024;                         // up to 16 z-bins x 256 centroids
constexpr int OFF_BAR = OFF_CB + 16 + CB_BYTES;             // 8-byte aligned below
constexpr int NBAR = 2 * STAGES + 1 + 2 + 2;                // full, empty, bfull, acc_full[2], acc_empty[2]
constexpr int OFF_TMEM = OFF_BAR + NBAR * 8 + 8;
constexpr int SMEM_BYTES = OFF_TMEM + 16 + 1024;            // + alignment slack of the 1024-byte base
constexpr int EPI_WARPS = 16;
constexpr int TRI = 8;                     // triplets per epilogue thread
constexpr int THREADS = (2 + EPI_WARPS) * 32;
constexpr int TMEM_COLS = 256;
// instruction descriptor: D f32 (bits 4-5 = 1), A bf16 (7-9 = 1), B bf16 (10-12 = 1), both K-major,
// N >> 3 at bits 17-22, M >> 4 at bits 24-28
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(D >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

// Shared-memory matrix descriptor of a K-major operand in the 64-byte swizzle
// layout: rows of 64 bytes, 8-row groups 512 bytes apart (stride byte offset),
// leading byte offset unused (1), version 1, layout type 4 (SWIZZLE_64B).
__device__ __forceinline__ uint64_t sw64_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(512u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)4u << 61);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        :: "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar) : "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.u32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(dtmem), "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate) : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 8 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    #pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    #pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

template <int CB>
__global__ void __launch_bounds__(THREADS, 1)
encode_tc_kernel(CodecArgs a, const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_r) {
    extern __shared__ uint8_t etc_smem_raw[];
    // 1024-byte aligned base for the swizzled operands, derived from the array itself (pointer plus
    // offset) so that every access below stays a shared-memory access
    uint8_t* smem = etc_smem_raw + ((1024u - (smem_u32(etc_smem_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    float* thr = reinterpret_cast<float*>(smem + OFF_THR);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + ((OFF_BAR + 7) & ~7));
    uint64_t* full = bars;
    uint64_t* empty = full + STAGES;
    uint64_t* bfull = empty + STAGES;
    uint64_t* acc_full = bfull + 1;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM);
    float2* cb_s = reinterpret_cast<float2*>(smem + ((OFF_CB + 15) & ~15));

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nz = (1 << a.bits_z) - 1, nr = (1 << a.bits_r) - 1, nt = (1 << a.bits_t) - 1;
    for (int i = tid; i < nz; i += THREADS) thr[i] = __ldg(a.z_thr + i);
    if (a.xy_mode == 0) {
        for (int i = tid; i < nr; i += THREADS) thr[nz + i] = __ldg(a.r2_thr + i);
        for (int i = tid; i < nt; i += THREADS) thr[nz + nr + i] = __ldg(a.th_thr + i);
    }
    const bool cb_in_smem = a.xy_mode == 1 && (int64_t)(nz + 1) * a.K * 8 <= CB_BYTES;
    __syncthreads();                        // thresholds in place for the guesses below
    if (cb_in_smem) {
        const float2* g = reinterpret_cast<const float2*>(a.codebook);
        for (int i = tid; i < (nz + 1) * a.K; i += THREADS) cb_s[i] = __ldg(g + i);
    }
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(bfull, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], EPI_WARPS);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int64_t ntiles = (a.n + BM - 1) / BM;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            mbar_arrive_expect_tx(bfull, NPART * B_PART);
            for (int p = 0; p < NPART; ++p)
                for (int c = 0; c < 3; ++c)
                    tma_load_2d(sbase + OFF_B + p * B_PART + c * B_CHUNK, &tmap_r, c * CHUNK_K, p * D,
                                smem_u32(bfull));
            int it = 0;
            bool ok = true;
            for (int64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
                const int s = it % STAGES;
                if (it >= STAGES && !mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, kErrWaitEmpty)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&full[s], A_TILE);
                for (int c = 0; c < 3; ++c)
                    tma_load_2d(sbase + OFF_A + s * A_TILE + c * A_CHUNK, &tmap_x, c * CHUNK_K, (int)(t * BM),
                                smem_u32(&full[s]));
            }
            // drain: every copy issued has landed before the CTA may exit
            mbar_wait(bfull, 0, kErrWaitDrain);
            for (int q = max(0, it - STAGES); q < it; ++q)
                mbar_wait(&full[q % STAGES], (q / STAGES) & 1, kErrWaitDrain);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            bool ok = mbar_wait(bfull, 0, kErrWaitFull);
            int it = 0, issued = 0;
            for (int64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
                const int s = it % STAGES, b = it & 1;
                if (!mbar_wait(&full[s], (it / STAGES) & 1, kErrWaitFull)) { ok = false; break; }
                if (it >= 2 && !mbar_wait(&acc_empty[b], ((it >> 1) - 1) & 1, kErrWaitEmpty)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(b * 128);
                #pragma unroll
                for (int p = 0; p < NPART; ++p) {
                    #pragma unroll
                    for (int k = 0; k < D / 16; ++k) {
                        const uint32_t koff = (uint32_t)((k >> 1) * A_CHUNK + (k & 1) * 32);
                        const uint32_t kofb = (uint32_t)((k >> 1) * B_CHUNK + (k & 1) * 32);
                        mma_bf16(d, sw64_desc(sbase + OFF_A + s * A_TILE + koff),
                                 sw64_desc(sbase + OFF_B + p * B_PART + kofb), (p | k) != 0);
                    }
                }
                mma_commit(smem_u32(&empty[s]));
                mma_commit(smem_u32(&acc_full[b]));
                issued = it + 1;
            }
            // the last accumulator's MMAs must be complete before tensor memory is freed
            if (issued > 0) mbar_wait(&acc_full[(issued - 1) & 1], ((issued - 1) >> 1) & 1, kErrWaitDrain);
        }
    } else {
        // ---------------- epilogue ----------------
        const int quarter = warp & 3, slice = (warp - 2) >> 2;      // TMEM lane quarter, 8-triplet slice
        const BinGuess guess = make_guess(thr, nz, nr, nt);
        const int row = quarter * 32 + lane;
        int it = 0;
        for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
            const int b = it & 1;
            // warp-uniform: tcgen05.ld below is .sync.aligned, so all lanes go on or none does
            // spin waits measured faster for the uniform-polar epilogue, the hinted wait for the
            // (longer) learned-codebook one
            const bool got = a.xy_mode == 0 ? mbar_wait_spin(&acc_full[b], (it >> 1) & 1, kErrWaitFull)
                                            : mbar_wait(&acc_full[b], (it >> 1) & 1, kErrWaitFull);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            float v[3 * TRI];
            const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * 128 + slice * 3 * TRI);
            tmem_ld16(taddr, *reinterpret_cast<float(*)[16]>(v));
            tmem_ld8(taddr + 16, v + 16);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
            const int64_t n = t * BM + row;
            if (n < a.n) {
                uint32_t c[TRI];
                #pragma unroll
                for (int j = 0; j < TRI; ++j)
                    c[j] = encode_triplet(a, thr, nz, nr, v[3 * j], v[3 * j + 1], v[3 * j + 2],
                                          cb_in_smem ? cb_s : nullptr, &guess);
                if (CB == 2) {
                    uint16_t* dst = static_cast<uint16_t*>(a.out) + code_row(a, n, a.out_stride) + TRI * slice;
                    const uint4 w = make_uint4(c[0] | (c[1] << 16), c[2] | (c[3] << 16), c[4] | (c[5] << 16),
                                               c[6] | (c[7] << 16));
                    if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                        *reinterpret_cast<uint4*>(dst) = w;
                    } else {
                        #pragma unroll
                        for (int j = 0; j < TRI; ++j) dst[j] = (uint16_t)c[j];
                    }
                } else {
                    uint8_t* dst = static_cast<uint8_t*>(a.out) + code_row(a, n, a.out_stride) + TRI * slice;
                    const uint2 w = make_uint2(c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24),
                                               c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24));
                    if ((reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
                        *reinterpret_cast<uint2*>(dst) = w;
                    } else {
                        #pragma unroll
                        for (int j = 0; j < TRI; ++j) dst[j] = (uint8_t)c[j];
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D bf16 tensor map: `rows` rows of 96 elements, `row_bytes` apart; boxes of
// 32 columns x box_rows rows in the 64-byte swizzle; rows past the end read 0.
static bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes, int box_rows) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)CHUNK_K, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace etc

// Tensor-core encode when it applies (head_dim 96, bf16 input rows 16-byte
// aligned, R parts present); PKV_ERR_UNSUPPORTED tells the caller to use the
// CUDA-core kernel.
int launch_encode_tc(const CodecArgs& a, int xdt, int cb, const void* r_bf16x3, cudaStream_t st) {
    using namespace etc;
    if (a.dim != D || xdt != PKV_BF16 || !r_bf16x3 || a.n <= 0) return PKV_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(a.in) & 15) || ((a.in_stride * 2) & 15)) return PKV_ERR_UNSUPPORTED;
    if (a.n > (int64_t)1 << 31) return PKV_ERR_UNSUPPORTED;     // TMA row coordinates are 32-bit
    if (cb != 1 && cb != 2) return PKV_ERR_UNSUPPORTED;
    CUtensorMap mx, mr;
    if (!make_map(&mx, a.in, a.n, a.in_stride * 2, BM)) return PKV_ERR_UNSUPPORTED;
    if (!make_map(&mr, r_bf16x3, NPART * D, D * 2, D)) return PKV_ERR_UNSUPPORTED;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                 cudaSuccess)
        return PKV_ERR_CUDA;
    const int64_t ntiles = (a.n + BM - 1) / BM;
    const int grid = (int)std::min<int64_t>(ntiles, sms);
    if (cb == 1) {
        if (cudaFuncSetAttribute(encode_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
            cudaSuccess)
            return PKV_ERR_CUDA;
        encode_tc_kernel<1><<<grid, THREADS, SMEM_BYTES, st>>>(a, mx, mr);
    } else {
        if (cudaFuncSetAttribute(encode_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
            cudaSuccess)
            return PKV_ERR_CUDA;
        encode_tc_kernel<2><<<grid, THREADS, SMEM_BYTES, st>>>(a, mx, mr);
    }
    return cudaGetLastError() == cudaSuccess ? PKV_OK : PKV_ERR_CUDA;
}

}  // namespace pkv
