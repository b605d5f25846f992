// pkv_scores.cu -- dense attention logits from packed key codes.
//
// Replaces prismkv_cuda.polar_attn_fwd (src/prismkv/cuda/prismkv_cuda.cpp:9-18,
// kernel polar_attn_kernel.cu:142-260): S[b,h,i,j] = scale * <Q_rot[b,h,i], k_j>
// for a query already rotated by R, with k_j the uniform-polar dequantization
// of the key codes.  The reference's kernel evaluates q_r*k_r*cos(q_theta -
// k_theta) per (i, j, triplet) with atan2/sqrt of the query recomputed for every
// key; here each 64-key tile is dequantized once into shared memory (the polar
// identity makes that exact: r cos(a - b) = x_q x_k + y_q y_k) and every
// query row reuses it.  Dequantization follows the reference fallback
// (cuda/__init__.py:64-92 -> polar_attention.py:153-171):
//   z = z_min + (i_z + 0.5) * delta_z,  r = i_r / (C_r - 1) * r_max,
//   theta = i_theta / (C_theta - 1) * 2 pi - pi,  (x, y) = r (cos, sin) theta.

#include "pkv_common.cuh"

namespace pkv {

constexpr int kScoreKeys = 64;

struct ScoreParams {
    const float* q; const uint8_t* kc; float* out;
    int B, H, Sq, Sk, dim, m, cb;
    int bits_z, bits_r, bits_t;
    float z_min, dz, r_max, two_pi, pi, scale;
};

template <int CB>
__global__ void __launch_bounds__(256) polar_scores_kernel(ScoreParams p) {
    using CT = typename Code<CB>::T;
    extern __shared__ float sm[];
    const int Cz = 1 << p.bits_z, Cr = 1 << p.bits_r, Ct = 1 << p.bits_t;
    float* tz = sm;                          // [Cz]
    float* tx = tz + Cz;                     // [Cr*Ct]
    float* ty = tx + Cr * Ct;
    const int pitch = (p.dim & 1) ? p.dim : p.dim + 1;
    float* kt = ty + Cr * Ct;                // [64][pitch]
    const int tid = threadIdx.x;
    for (int i = tid; i < Cz; i += blockDim.x)
        tz[i] = __fadd_rn(p.z_min, __fmul_rn(__fadd_rn((float)i, 0.5f), p.dz));
    for (int i = tid; i < Cr * Ct; i += blockDim.x) {
        const int ir = i / Ct, it = i % Ct;
        const float r = __fmul_rn(__fdiv_rn((float)ir, (float)max(Cr - 1, 1)), p.r_max);
        const float th = __fsub_rn(__fmul_rn(__fdiv_rn((float)it, (float)max(Ct - 1, 1)), p.two_pi), p.pi);
        tx[i] = __fmul_rn(r, cosf(th));
        ty[i] = __fmul_rn(r, sinf(th));
    }
    __syncthreads();
    const int bh = blockIdx.x;
    const int j0 = blockIdx.y * kScoreKeys;
    const CT* codes = reinterpret_cast<const CT*>(p.kc) + ((int64_t)bh * p.Sk) * p.m;
    const uint32_t flat_bits = p.bits_r + p.bits_t;
    const uint32_t mask = (1u << (p.bits_z + flat_bits)) - 1u;
    for (int idx = tid; idx < kScoreKeys * p.m; idx += blockDim.x) {
        const int jj = idx / p.m, t = idx % p.m;
        const int j = j0 + jj;
        float z = 0.f, x = 0.f, y = 0.f;
        if (j < p.Sk) {
            const uint32_t c = Code<CB>::load(codes + (int64_t)j * p.m + t) & mask;
            z = tz[c >> flat_bits];
            x = tx[c & ((1u << flat_bits) - 1u)];
            y = ty[c & ((1u << flat_bits) - 1u)];
        }
        kt[jj * pitch + 3 * t] = z;
        kt[jj * pitch + 3 * t + 1] = x;
        kt[jj * pitch + 3 * t + 2] = y;
    }
    __syncthreads();
    const int jj = tid % kScoreKeys, qg = tid / kScoreKeys;
    const int j = j0 + jj;
    const float* qb = p.q + (int64_t)bh * p.Sq * p.dim;
    for (int i = qg; i < p.Sq; i += blockDim.x / kScoreKeys) {
        const float* qr = qb + (int64_t)i * p.dim;
        float acc = 0.f;
        #pragma unroll 4
        for (int k = 0; k < p.dim; ++k) acc = fmaf(__ldg(qr + k), kt[jj * pitch + k], acc);
        if (j < p.Sk) p.out[((int64_t)bh * p.Sq + i) * p.Sk + j] = p.scale * acc;
    }
}

int launch_polar_scores(const float* q, const void* kc, int cb, int B, int H, int Sq, int Sk, int dim,
                        const float* qp, const int32_t* bits, float* out, cudaStream_t st) {
    ScoreParams p{};
    p.q = q; p.kc = static_cast<const uint8_t*>(kc); p.out = out;
    p.B = B; p.H = H; p.Sq = Sq; p.Sk = Sk; p.dim = dim; p.m = dim / 3; p.cb = cb;
    p.bits_z = bits[0]; p.bits_r = bits[1]; p.bits_t = bits[2];
    // z_max = z_min + delta_z * C_z and delta_z = (z_max - z_min) / C_z, in double
    // as the reference fallback does (cuda/__init__.py:82-83, polar_attention.py:166).
    const double Cz = (double)(1 << bits[0]);
    const double z_min = qp[0], z_max = z_min + (double)qp[1] * Cz;
    p.z_min = (float)z_min;
    p.dz = (float)((z_max - z_min) / Cz);
    p.r_max = qp[2];
    p.two_pi = (float)(2.0 * 3.141592653589793);
    p.pi = (float)3.141592653589793;
    p.scale = qp[5];
    if ((int64_t)B * H * Sq * Sk == 0) return PKV_OK;
    const int pitch = (dim & 1) ? dim : dim + 1;
    const size_t smem = sizeof(float) * ((1 << bits[0]) + 2 * (1 << (bits[1] + bits[2])) + kScoreKeys * pitch);
    if ((Sk + kScoreKeys - 1) / kScoreKeys > 65535) return PKV_ERR_UNSUPPORTED;
    dim3 grid(B * H, (Sk + kScoreKeys - 1) / kScoreKeys);
    if (cb == 1) {
        if (smem > 48 * 1024 &&
            cudaFuncSetAttribute(polar_scores_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return PKV_ERR_CUDA;
        polar_scores_kernel<1><<<grid, 256, smem, st>>>(p);
    } else {
        if (smem > 48 * 1024 &&
            cudaFuncSetAttribute(polar_scores_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return PKV_ERR_CUDA;
        polar_scores_kernel<2><<<grid, 256, smem, st>>>(p);
    }
    return cudaGetLastError() == cudaSuccess ? PKV_OK : PKV_ERR_CUDA;
}

}  // namespace pkv
