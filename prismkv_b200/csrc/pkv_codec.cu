// pkv_codec.cu -- encode (rotate + bin + pack) and decode (LUT + un-rotate).
//
// Encode restates StackedPlaneQuantizer.encode (stacked_plane.py:210-262):
//   rot = x @ R^T ; z -> i_z (uniform floor bins or Lloyd-Max bucketize) ;
//   (x, y) -> (i_r, i_theta) on the uniform polar grid, or the nearest
//   learned centroid of bin i_z (learned_codebook.py:217-248) ;
//   code = i_z << (bits_r + bits_theta) | i_flat.
// The fp32 chains that follow the rotation in the reference ((z - z_min) /
// delta_z -> floor -> clamp, sqrt -> clamp -> / r_max * (C-1) -> round, ...)
// are monotone in their input, so each is replaced by an exact count of
// host-computed thresholds on the same fp32 input (z, x*x + y*y, atan2).
//
// Decode restates StackedPlaneQuantizer.decode (stacked_plane.py:268-327):
// table lookup of the dequantized (z, x, y) triplet (BiasTable folded into
// the table on the host), then rot_q @ R.
//
// Both run one CTA per 64*RPT rows; the 96x96 (generally dim x dim) GEMM is
// register-blocked on CUDA cores with R staged in shared memory.

#include <algorithm>

#include "pkv_common.cuh"

namespace pkv {


struct CodecArgs {
    int dim, m, kp;            // kp: padded column count of the staged matrix (12*MPT)
    int bits_z, bits_r, bits_t, bits_flat, K;
    int xy_mode, xy_per_z, z_nan_bin;
    float z_hi;
    const float* R;
    const float* z_thr;
    const float* r2_thr;
    const float* th_thr;
    const float* codebook;
    const float* dec_z;
    const float* dec_xy;
    const void* in;            // x (encode) or codes (decode)
    void* out;                 // codes (encode) or vectors (decode)
    int64_t n, in_stride, out_stride;
    // learned codebooks: candidate centroids per grid cell (cell_grid 0 = scan all K)
    const uint8_t* cell_idx;
    const uint8_t* cell_cnt;
    int cell_grid;
    float cell_lo, cell_scale;             // cell = floor((v - cell_lo) * cell_scale)
    // code rows grouped as in a KV cache (0 = plain rows): code row n sits at
    // (n / group_rows) * group_stride + (n % group_rows) * stride, in codes
    int64_t group_rows, group_stride;
};

__device__ __forceinline__ int64_t code_row(const CodecArgs& a, int64_t n, int64_t stride) {
    return a.group_rows > 0 ? (n / a.group_rows) * a.group_stride + (n % a.group_rows) * stride : n * stride;
}

// acc[rr][c] += sum_i A[row_rr][i] * B[i][col0 + c]    (A: [TR][lda], B: [K][kp])
template <int MPT, int RPT>
__device__ __forceinline__ void tile_gemm(const float* __restrict__ As, int lda,
                                          const float* __restrict__ Bs, int kp, int kdim,
                                          int row0, int col0, float (&acc)[RPT][3 * MPT]) {
    #pragma unroll
    for (int rr = 0; rr < RPT; ++rr)
        #pragma unroll
        for (int c = 0; c < 3 * MPT; ++c) acc[rr][c] = 0.f;
    #pragma unroll 2
    for (int i = 0; i < kdim; ++i) {
        float xv[RPT];
        #pragma unroll
        for (int rr = 0; rr < RPT; ++rr) xv[rr] = As[(row0 + 64 * rr) * lda + i];
        const float4* b4 = reinterpret_cast<const float4*>(Bs + i * kp + col0);
        #pragma unroll
        for (int c4 = 0; c4 < (3 * MPT) / 4; ++c4) {
            float4 bv = b4[c4];
            #pragma unroll
            for (int rr = 0; rr < RPT; ++rr) {
                acc[rr][4 * c4 + 0] = fmaf(xv[rr], bv.x, acc[rr][4 * c4 + 0]);
                acc[rr][4 * c4 + 1] = fmaf(xv[rr], bv.y, acc[rr][4 * c4 + 1]);
                acc[rr][4 * c4 + 2] = fmaf(xv[rr], bv.z, acc[rr][4 * c4 + 2]);
                acc[rr][4 * c4 + 3] = fmaf(xv[rr], bv.w, acc[rr][4 * c4 + 3]);
            }
        }
    }
}

// Nearest learned centroid (learned_codebook.py:217-248).  Finite points:
// first index of the minimal squared distance.  A point with an infinite
// coordinate follows cdist's matrix-product form -2p.c + |p|^2 + |c|^2,
// whose result per centroid is NaN or +inf; argmin takes the first NaN,
// else index 0.  A NaN point gives 0.
__device__ __forceinline__ int nearest_centroid(const float2* __restrict__ cb, int K, float x, float y) {
    if (isfinite(x) && isfinite(y)) {
        float best = INFINITY;
        int bi = 0;
        #pragma unroll 4
        for (int k = 0; k < K; ++k) {
            float2 c = __ldg(cb + k);
            float dx = x - c.x, dy = y - c.y;
            float d2 = fmaf(dx, dx, dy * dy);
            if (d2 < best) { best = d2; bi = k; }
        }
        return bi;
    }
    if (isnan(x) || isnan(y)) return 0;
    float pn = __fadd_rn(__fmul_rn(x, x), __fmul_rn(y, y));
    for (int k = 0; k < K; ++k) {
        float2 c = __ldg(cb + k);
        float t = __fadd_rn(__fmul_rn(__fmul_rn(-2.f, x), c.x), __fmul_rn(__fmul_rn(-2.f, y), c.y));
        t = __fadd_rn(__fadd_rn(t, pn), __fadd_rn(__fmul_rn(c.x, c.x), __fmul_rn(c.y, c.y)));
        if (isnan(t)) return k;
    }
    return 0;
}

// The same argmin over the candidate list of the point's grid cell: candidates
// are stored in ascending index order and include every centroid that can be
// (or tie with) the nearest for any point of the cell, so the result equals the
// full scan's.  Points outside the grid or in an overfull cell scan all K.
constexpr int kCellMax = 16;

// cb: bin iz's centroids in global memory; cb_fast: the same centroids where
// they are cheaper to read (a shared-memory copy), or cb itself.
__device__ __forceinline__ int nearest_centroid_cells(const CodecArgs& a, int iz, const float2* __restrict__ cb,
                                                      const float2* cb_fast, float x, float y) {
    if (a.cell_grid > 0 && isfinite(x) && isfinite(y)) {
        const float fx = (x - a.cell_lo) * a.cell_scale, fy = (y - a.cell_lo) * a.cell_scale;
        if (fx >= 0.f && fy >= 0.f && fx < (float)a.cell_grid && fy < (float)a.cell_grid) {
            const int cell = (iz * a.cell_grid + (int)fy) * a.cell_grid + (int)fx;
            // the count and the cell's candidate row (one 16-byte load) are fetched together
            static_assert(kCellMax == 16, "one 16-byte row per cell");
            const int n = __ldg(a.cell_cnt + cell);
            const uint4 row = __ldg(reinterpret_cast<const uint4*>(a.cell_idx) + cell);
            if (n <= kCellMax) {
                // scan in list (ascending index) order; a strict compare keeps the first minimum
                const uint32_t w4[4] = {row.x, row.y, row.z, row.w};
                float best = INFINITY;
                int bi = 0;
                #pragma unroll
                for (int i = 0; i < kCellMax; ++i) {
                    if (i < n) {
                        const int k = (int)((w4[i >> 2] >> (8 * (i & 3))) & 0xFFu);
                        const float2 c = cb_fast[k];
                        const float dx = x - c.x, dy = y - c.y;
                        const float d2 = fmaf(dx, dx, dy * dy);
                        if (d2 < best) { best = d2; bi = k; }
                    }
                }
                return bi;
            }
        }
    }
    return nearest_centroid(cb, a.K, x, y);
}

// Code of one rotated triplet (z, x, y): z bin by threshold count (NaN and
// values >= z_hi as the reference's chain maps them), then the uniform polar
// bins (r^2 and atan2 thresholds) or the nearest learned centroid of bin i_z.
// thr: z | r^2 | theta thresholds, nz = 2^bits_z - 1, nr = 2^bits_r - 1.
// cb_smem: the whole codebook in shared memory, or nullptr.  g (optional):
// linear first guesses of the three threshold counts (BinGuess), which replace
// the binary searches by one or two comparisons.
struct BinGuess {
    float z0, zi, r0, ri, t0, ti;          // count ~ floor((f(v) - x0) * xi) + 1, f = sqrt for r^2
};

__device__ __forceinline__ BinGuess make_guess(const float* thr, int nz, int nr, int nt) {
    auto lin = [](const float* t, int n, bool root, float& x0, float& xi) {
        const float lo = root ? sqrtf(t[0]) : t[0], hi = root ? sqrtf(t[n - 1]) : t[n - 1];
        x0 = lo;
        xi = (n > 1 && hi > lo) ? (float)(n - 1) / (hi - lo) : 0.f;
    };
    BinGuess g;
    lin(thr, nz, false, g.z0, g.zi);
    lin(thr + nz, nr, true, g.r0, g.ri);
    lin(thr + nz + nr, nt, false, g.t0, g.ti);
    return g;
}

// sqrt for a first guess only (hardware approximation, relative error ~2^-23; 0, +inf and NaN
// map to themselves): the exact r^2 threshold count around the guess decides the bin
__device__ __forceinline__ float guess_sqrt(float v) {
    float r;
    asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}

__device__ __forceinline__ int guess_count(float v, float x0, float xi) {
    return __float2int_rd(fmaf(v - x0, xi, 1.f));  // saturating (no overflow at +-inf); NaN gives 0
}

__device__ __forceinline__ uint32_t encode_triplet(const CodecArgs& a, const float* thr, int nz, int nr, float z,
                                                   float xx, float yy, const float2* cb_smem = nullptr,
                                                   const BinGuess* g = nullptr) {
    int iz;
    if (g) {
        // uniform z bins: the linear guess is within one bin; Lloyd-Max (z_hi NaN): binary search
        const int c = isnan(a.z_hi) ? count_ge_unrolled(thr, a.bits_z, z)
                                    : count_ge_window(thr, nz, z, guess_count(z, g->z0, g->zi));
        iz = isnan(z) ? a.z_nan_bin : (z >= a.z_hi ? 0 : c);
    } else {
        if (isnan(z)) iz = a.z_nan_bin;
        else if (z >= a.z_hi) iz = 0;
        else iz = count_ge(thr, a.bits_z, z);
    }
    uint32_t flat;
    if (a.xy_mode == 0) {
        float s = __fadd_rn(__fmul_rn(xx, xx), __fmul_rn(yy, yy));
        const float th = atan2f(yy, xx);
        const int nt = (1 << a.bits_t) - 1;
        int ir, it;
        if (g) {
            ir = count_ge_window(thr + nz, nr, s, guess_count(guess_sqrt(s), g->r0, g->ri));
            it = count_ge_window(thr + nz + nr, nt, th, guess_count(th, g->t0, g->ti));
        } else {
            ir = count_ge(thr + nz, a.bits_r, s);
            it = count_ge(thr + nz + nr, a.bits_t, th);
        }
        flat = ((uint32_t)ir << a.bits_t) | (uint32_t)it;
    } else {
        const float2* cb = reinterpret_cast<const float2*>(a.codebook) + (size_t)iz * a.K;
        flat = (uint32_t)nearest_centroid_cells(a, iz, cb, cb_smem ? cb_smem + (size_t)iz * a.K : cb, xx, yy);
    }
    return ((uint32_t)iz << a.bits_flat) | flat;
}

template <int MPT, int RPT, int XDT, int CB>
__global__ void __launch_bounds__(256) encode_kernel(CodecArgs a) {
    constexpr int TR = 64 * RPT;
    extern __shared__ __align__(16) float smem[];
    const int lda = (a.dim & 1) ? a.dim : a.dim + 1;   // odd row pitch: conflict-free column reads
    float* Bs = smem;                               // Rt: [dim][kp], Bs[i][k] = R[k][i]
    float* As = Bs + a.dim * a.kp;                  // [TR][dim+1]
    float* thr = As + TR * lda;                     // z | r2 | th thresholds
    const int nz = (1 << a.bits_z) - 1, nr = (1 << a.bits_r) - 1, nt = (1 << a.bits_t) - 1;

    const int tid = threadIdx.x;
    for (int idx = tid; idx < a.dim * a.kp; idx += blockDim.x) {
        int i = idx / a.kp, k = idx % a.kp;
        Bs[idx] = (k < a.dim) ? __ldg(a.R + k * a.dim + i) : 0.f;
    }
    for (int idx = tid; idx < nz; idx += blockDim.x) thr[idx] = __ldg(a.z_thr + idx);
    if (a.xy_mode == 0) {
        for (int idx = tid; idx < nr; idx += blockDim.x) thr[nz + idx] = __ldg(a.r2_thr + idx);
        for (int idx = tid; idx < nt; idx += blockDim.x) thr[nz + nr + idx] = __ldg(a.th_thr + idx);
    }
    __syncthreads();

    const int warp = tid >> 5, lane = tid & 31;
    const int row0 = (warp & 1) * 32 + lane;
    const int tg = warp >> 1;
    const int j0 = tg * MPT;
    using XT = typename Elem<XDT>::T;
    const XT* x = static_cast<const XT*>(a.in);
    using CT = typename Code<CB>::T;
    CT* codes = static_cast<CT*>(a.out);

    for (int64_t n0 = (int64_t)blockIdx.x * TR; n0 < a.n; n0 += (int64_t)gridDim.x * TR) {
        for (int idx = tid; idx < TR * a.dim; idx += blockDim.x) {
            int r = idx / a.dim, i = idx % a.dim;
            int64_t n = n0 + r;
            As[r * lda + i] = (n < a.n) ? Elem<XDT>::load(x + n * a.in_stride + i) : 0.f;
        }
        __syncthreads();
        float acc[RPT][3 * MPT];
        if (j0 < a.m) tile_gemm<MPT, RPT>(As, lda, Bs, a.kp, a.dim, row0, 3 * j0, acc);
        __syncthreads();
        if (j0 < a.m) {
            #pragma unroll
            for (int rr = 0; rr < RPT; ++rr) {
                int64_t n = n0 + row0 + 64 * rr;
                if (n >= a.n) continue;
                CT* crow = codes + code_row(a, n, a.out_stride);
                #pragma unroll
                for (int jj = 0; jj < MPT; ++jj) {
                    int j = j0 + jj;
                    if (j >= a.m) break;
                    Code<CB>::store(crow + j, encode_triplet(a, thr, nz, nr, acc[rr][3 * jj], acc[rr][3 * jj + 1],
                                                             acc[rr][3 * jj + 2]));
                }
            }
        }
    }
}

template <int MPT, int RPT, int CB, int ODT>
__global__ void __launch_bounds__(256) decode_kernel(CodecArgs a) {
    constexpr int TR = 64 * RPT;
    extern __shared__ __align__(16) float smem[];
    const int lda = (a.dim & 1) ? a.dim : a.dim + 1;
    float* Bs = smem;                               // R: [dim][kp], Bs[k][i] = R[k][i]
    float* As = Bs + a.dim * a.kp;                  // rotated triplets [TR][dim+1]
    const int tid = threadIdx.x;
    for (int idx = tid; idx < a.dim * a.kp; idx += blockDim.x) {
        int k = idx / a.kp, i = idx % a.kp;
        Bs[idx] = (i < a.dim) ? __ldg(a.R + k * a.dim + i) : 0.f;
    }
    __syncthreads();
    const int warp = tid >> 5, lane = tid & 31;
    const int row0 = (warp & 1) * 32 + lane;
    const int tg = warp >> 1;
    const int j0 = tg * MPT;
    using CT = typename Code<CB>::T;
    const CT* codes = static_cast<const CT*>(a.in);
    using OT = typename Elem<ODT>::T;
    OT* out = static_cast<OT*>(a.out);
    const uint32_t mask = (1u << (a.bits_z + a.bits_flat)) - 1u;
    const uint32_t fmask = (1u << a.bits_flat) - 1u;
    const float2* dxy = reinterpret_cast<const float2*>(a.dec_xy);

    for (int64_t n0 = (int64_t)blockIdx.x * TR; n0 < a.n; n0 += (int64_t)gridDim.x * TR) {
        for (int idx = tid; idx < TR * a.m; idx += blockDim.x) {
            int r = idx / a.m, j = idx % a.m;
            int64_t n = n0 + r;
            float z = 0.f, xx = 0.f, yy = 0.f;
            if (n < a.n) {
                uint32_t c = Code<CB>::load(codes + code_row(a, n, a.in_stride) + j) & mask;
                z = __ldg(a.dec_z + (c >> a.bits_flat));
                float2 xy = __ldg(dxy + (a.xy_per_z ? c : (c & fmask)));
                xx = xy.x; yy = xy.y;
            }
            As[r * lda + 3 * j] = z;
            As[r * lda + 3 * j + 1] = xx;
            As[r * lda + 3 * j + 2] = yy;
        }
        __syncthreads();
        float acc[RPT][3 * MPT];
        if (j0 < a.m) tile_gemm<MPT, RPT>(As, lda, Bs, a.kp, a.dim, row0, 3 * j0, acc);
        __syncthreads();
        if (j0 < a.m) {
            #pragma unroll
            for (int rr = 0; rr < RPT; ++rr) {
                int64_t n = n0 + row0 + 64 * rr;
                if (n >= a.n) continue;
                #pragma unroll
                for (int c = 0; c < 3 * MPT; ++c) {
                    int col = 3 * j0 + c;
                    if (col < a.dim) Elem<ODT>::store(out + n * a.out_stride + col, acc[rr][c]);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------

static int sm_count() {
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

template <typename KernelT>
static int launch_persistent(KernelT kern, size_t smem, int64_t tiles, const CodecArgs& a, cudaStream_t st) {
    if (smem > 48 * 1024) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return PKV_ERR_CUDA;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, smem) != cudaSuccess || per_sm <= 0)
        return PKV_ERR_CUDA;
    int64_t grid = std::min<int64_t>(tiles, (int64_t)per_sm * sm_count());
    kern<<<(unsigned)grid, 256, smem, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? PKV_OK : PKV_ERR_CUDA;
}

template <int MPT, int RPT, int XDT>
static int encode_dispatch_cb(const CodecArgs& a, int cb, size_t smem, int64_t tiles, cudaStream_t st) {
    switch (cb) {
        case 1: return launch_persistent(encode_kernel<MPT, RPT, XDT, 1>, smem, tiles, a, st);
        case 2: return launch_persistent(encode_kernel<MPT, RPT, XDT, 2>, smem, tiles, a, st);
        case 8: return launch_persistent(encode_kernel<MPT, RPT, XDT, 8>, smem, tiles, a, st);
    }
    return PKV_ERR_INVALID;
}

template <int MPT, int RPT>
static int encode_dispatch(const CodecArgs& a, int xdt, int cb, cudaStream_t st) {
    constexpr int TR = 64 * RPT;
    size_t smem = sizeof(float) * ((size_t)a.dim * a.kp + (size_t)TR * (a.dim + 1) + 3 * 256);
    int64_t tiles = (a.n + TR - 1) / TR;
    switch (xdt) {
        case PKV_F32: return encode_dispatch_cb<MPT, RPT, PKV_F32>(a, cb, smem, tiles, st);
        case PKV_BF16: return encode_dispatch_cb<MPT, RPT, PKV_BF16>(a, cb, smem, tiles, st);
        case PKV_F16: return encode_dispatch_cb<MPT, RPT, PKV_F16>(a, cb, smem, tiles, st);
    }
    return PKV_ERR_INVALID;
}

template <int MPT, int RPT, int CB>
static int decode_dispatch_odt(const CodecArgs& a, int odt, size_t smem, int64_t tiles, cudaStream_t st) {
    switch (odt) {
        case PKV_F32: return launch_persistent(decode_kernel<MPT, RPT, CB, PKV_F32>, smem, tiles, a, st);
        case PKV_BF16: return launch_persistent(decode_kernel<MPT, RPT, CB, PKV_BF16>, smem, tiles, a, st);
        case PKV_F16: return launch_persistent(decode_kernel<MPT, RPT, CB, PKV_F16>, smem, tiles, a, st);
    }
    return PKV_ERR_INVALID;
}

template <int MPT, int RPT>
static int decode_dispatch(const CodecArgs& a, int cb, int odt, cudaStream_t st) {
    constexpr int TR = 64 * RPT;
    size_t smem = sizeof(float) * ((size_t)a.dim * a.kp + (size_t)TR * (a.dim + 1));
    int64_t tiles = (a.n + TR - 1) / TR;
    switch (cb) {
        case 1: return decode_dispatch_odt<MPT, RPT, 1>(a, odt, smem, tiles, st);
        case 2: return decode_dispatch_odt<MPT, RPT, 2>(a, odt, smem, tiles, st);
        case 8: return decode_dispatch_odt<MPT, RPT, 8>(a, odt, smem, tiles, st);
    }
    return PKV_ERR_INVALID;
}

static void fill_args(CodecArgs& a, const pkv_codec* c) {
    a.dim = c->dim;
    a.m = c->dim / 3;
    a.bits_z = c->bits_z; a.bits_r = c->bits_r; a.bits_t = c->bits_theta;
    a.bits_flat = c->bits_r + c->bits_theta;
    a.K = 1 << a.bits_flat;
    a.xy_mode = c->xy_mode; a.xy_per_z = c->xy_per_z; a.z_nan_bin = c->z_nan_bin;
    a.z_hi = c->z_hi;
    a.R = c->R; a.z_thr = c->z_thr; a.r2_thr = c->r2_thr; a.th_thr = c->th_thr;
    a.codebook = c->codebook; a.dec_z = c->dec_z; a.dec_xy = c->dec_xy;
    a.cell_grid = 0;
    // each cell's 16-entry candidate row is read with one 16-byte load: a table that is not
    // 16-byte aligned takes the full scan instead
    if (c->xy_mode == 1 && c->cell_idx && c->cell_cnt && c->cell_grid > 0 && c->cell_half_width > 0.f &&
        (reinterpret_cast<uintptr_t>(c->cell_idx) & 15u) == 0 && (1 << (c->bits_r + c->bits_theta)) <= 256) {
        a.cell_idx = c->cell_idx;
        a.cell_cnt = c->cell_cnt;
        a.cell_grid = c->cell_grid;
        a.cell_lo = -c->cell_half_width;
        a.cell_scale = (float)c->cell_grid / (2.f * c->cell_half_width);
    }
}

int launch_encode_tc(const CodecArgs& a, int xdt, int cb, const void* r_bf16x3, cudaStream_t st);

int launch_encode(const pkv_codec* c, const void* x, int xdt, int64_t n, int64_t xs,
                  void* codes, int cb, int64_t cs, int64_t group_rows, int64_t group_stride, cudaStream_t st) {
    CodecArgs a{};
    fill_args(a, c);
    a.in = x; a.out = codes; a.n = n; a.in_stride = xs; a.out_stride = cs;
    a.group_rows = group_rows; a.group_stride = group_stride;
    const int rc = launch_encode_tc(a, xdt, cb, c->R_bf16x3, st);     // tensor cores where they apply
    if (rc != PKV_ERR_UNSUPPORTED) return rc;
    if (a.m <= 32) { a.kp = 96; return encode_dispatch<8, 2>(a, xdt, cb, st); }
    a.kp = 192;
    return encode_dispatch<16, 1>(a, xdt, cb, st);
}

int launch_decode(const pkv_codec* c, const void* codes, int cb, int64_t n, int64_t cs,
                  void* out, int odt, int64_t os, int64_t group_rows, int64_t group_stride, cudaStream_t st) {
    CodecArgs a{};
    fill_args(a, c);
    a.in = codes; a.out = out; a.n = n; a.in_stride = cs; a.out_stride = os;
    a.group_rows = group_rows; a.group_stride = group_stride;
    if (a.m <= 32) { a.kp = 96; return decode_dispatch<8, 2>(a, cb, odt, st); }
    a.kp = 192;
    return decode_dispatch<16, 1>(a, cb, odt, st);
}

}  // namespace pkv
