/*
 * prismkv_b200.h -- C ABI of the B200 (sm_100a) PrismKV quantized-KV hot path.
 *
 * Every entry point takes plain device pointers, element counts, strides and
 * a CUDA stream (passed as `void *`, it is a `cudaStream_t`), returns an int
 * status (0 = PKV_OK) and allocates no device memory (pkv_xr_alloc, the
 * one-time set-up of the split-sequence exchange, is the exception).  Buffers are owned
 * by the caller.  Kernels are enqueued on the given stream; no entry point
 * synchronises the host.  Entry points are re-entrant: concurrent calls on
 * different streams are safe as long as they do not share a workspace.
 *
 * Units: dim = head dimension d (a multiple of 3), m = dim / 3 triplets,
 * codes are packed (i_z << (bits_r + bits_theta)) | i_flat.
 *
 * Reference interfaces replaced (PrismKV v1.4.1, paths inside that project):
 *   pkv_encode         StackedPlaneQuantizer.encode   src/prismkv/quantizer/stacked_plane.py:210-262
 *                      (+ LearnedSliceCodebook.encode_xy learned_codebook.py:217-248,
 *                         LloydMaxQuantizer1D.encode lloyd_max.py:106-124)
 *   pkv_decode         StackedPlaneQuantizer.decode   src/prismkv/quantizer/stacked_plane.py:268-327
 *                      (+ decode_xy learned_codebook.py:250-269, BiasTable.apply
 *                         bias_correction.py:58-91, LloydMaxQuantizer1D.decode lloyd_max.py:126-140)
 *   pkv_attn_decode    PolarAttentionApprox.forward   src/prismkv/quantizer/polar_attention.py:277-309
 *                      fused with decode of V; no reference kernel exists
 *   pkv_polar_scores   prismkv_cuda.polar_attn_fwd    src/prismkv/cuda/prismkv_cuda.cpp:9-18,
 *                      kernel src/prismkv/cuda/polar_attn_kernel.cu:142-336,
 *                      Python contract src/prismkv/cuda/__init__.py:23-61
 *   pkv_lse_combine    (new) log-sum-exp merge of split-sequence partials
 *   pkv_attn_decode_xr (new) split-sequence decode with the cross-GPU merge
 *                      inside the attention kernel (pkv_xr_* set it up)
 */
#ifndef PRISMKV_B200_H
#define PRISMKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PKV_ABI_VERSION 1

#if defined(__GNUC__)
#define PKV_API __attribute__((visibility("default")))
#else
#define PKV_API
#endif

/* ---- status codes ------------------------------------------------------ */
enum {
    PKV_OK = 0,
    PKV_ERR_INVALID = 1,      /* null pointer, bad shape, bits out of range      */
    PKV_ERR_UNSUPPORTED = 2,  /* well-formed but outside what this library runs  */
    PKV_ERR_ALIGNMENT = 3,    /* pointer or stride misaligned for the call       */
    PKV_ERR_WORKSPACE = 4,    /* workspace missing or smaller than required      */
    PKV_ERR_CUDA = 5,         /* CUDA runtime reported an error (launch/config)  */
    PKV_ERR_DEVICE = 6,       /* a kernel flagged an error (bounded wait expired)*/
    PKV_ERR_SCRATCH_LIMIT = 7 /* pkv_attn_decode_noalloc: needs more scratch than
                                 its static array holds                          */
};

/* ---- codec flags -------------------------------------------------------- */
#define PKV_CODEC_Z_UNIFORM 1   /* uniform z bins without BiasTable (dec_z affine in i_z) */
#define PKV_CODEC_FP32_ATTN 2   /* attention arithmetic in fp32 throughout: no fp16-pair
                                   tensor-core tiles (attn_gqa12_mma_kernel is not planned) */

/* ---- element types ----------------------------------------------------- */
enum { PKV_F32 = 0, PKV_BF16 = 1, PKV_F16 = 2 };

/* ---- quantizer state ---------------------------------------------------- *
 * All table pointers are device pointers.  Tables are built on the host
 * once per quantizer (they are the quantizer's parameters, not data):
 *   z_thr    (2^bits_z - 1)   i_z  = #{b : z >= z_thr[b]}            (ascending)
 *   r2_thr   (2^bits_r - 1)   i_r  = #{b : x*x + y*y >= r2_thr[b]}   (polar path)
 *   th_thr   (2^bits_theta-1) i_th = #{b : atan2(y, x) >= th_thr[b]} (polar path)
 *   codebook (2^bits_z, K, 2) learned (x, y) centroids, K = 2^(bits_r+bits_theta)
 *   dec_z    (2^bits_z)       dequantized z per bin, BiasTable folded in
 *   dec_xy   (xy_per_z ? 2^bits_z * K : K, 2) dequantized (x, y), bias folded in
 *   bias_xy  (2^bits_z, 2) the clamped BiasTable (x, y) terms alone (NULL when
 *            there is no BiasTable); the polar attention path subtracts them
 *            per z-bin instead of reading the per-code dec_xy
 * z_hi: z >= z_hi maps to bin 0 (uniform bins: the reference's int64
 * conversion of an out-of-range floor); NaN when unused.  z_nan_bin: bin of
 * a NaN z (0 for uniform bins, 2^bits_z - 1 for Lloyd-Max boundaries).     */
typedef struct pkv_codec {
    int32_t dim;
    int32_t bits_z, bits_r, bits_theta;   /* each 1..8, sum <= 16            */
    int32_t xy_mode;                      /* 0 uniform polar, 1 codebook     */
    int32_t xy_per_z;                     /* dec_xy indexed by full code     */
    int32_t z_nan_bin;
    float z_hi;
    float r_max;                          /* polar grid: r(i_r) = i_r * r_max / (2^bits_r - 1) */
    int32_t flags;                        /* PKV_CODEC_Z_UNIFORM: dec_z[i] = dec_z[0] + i * step */
    const float *R;                       /* (dim, dim) row-major rotation   */
    const float *z_thr;
    const float *r2_thr;
    const float *th_thr;
    const float *codebook;
    const float *dec_z;
    const float *dec_xy;
    const float *bias_xy;                 /* (2^bits_z, 2) clamped BiasTable (x, y), or NULL */
    /* Learned codebooks, optional: candidate centroids per cell of a
     * cell_grid x cell_grid grid over [-cell_half_width, cell_half_width]^2
     * per z-bin (cell_idx [2^bits_z][grid][grid][16] ascending indices,
     * cell_cnt [2^bits_z][grid][grid], 255 = scan all).  NULL, or a
     * cell_idx that is not 16-byte aligned: full scan.                       */
    const uint8_t *cell_idx;
    const uint8_t *cell_cnt;
    int32_t cell_grid;
    float cell_half_width;
    /* Optional: R as three bf16 parts (3, dim, dim), R ~= R1 + R2 + R3 with
     * R1 = bf16(R), R2 = bf16(R - R1), R3 = bf16(R - R1 - R2).  When set, bf16
     * inputs of head_dim 96 are rotated on the tensor cores.                */
    const void *R_bf16x3;
} pkv_codec;

/* ---- decode attention -------------------------------------------------- *
 * out[b, h, :] = softmax(q'[b,h] . Khat^T * scale) . Vhat  @ R
 * with q' = q @ R^T, Khat/Vhat the rotated-space dequantized codes, and
 * KV head h / (q_heads / kv_heads) serving query head h (grouped heads).
 * Codes live at k_codes + b*kv_batch_stride + hk*kv_head_stride + t*m (in
 * code units), t < seq_lens[b] (or seq_len when seq_lens is NULL).
 * partial_only != 0: write, per (b, h), the unnormalised rotated-space
 * partial [m_max, l, o[0..dim-1]] (natural-log max of score*scale,
 * l = sum exp(s - m_max), o = sum exp(s - m_max) * Vhat) to
 * partial_out + (b*q_heads + h) * (dim + 2), instead of out.                */
typedef struct pkv_attn_args {
    int32_t batch, q_heads, kv_heads, seq_len;
    const void *q;                 /* (batch, q_heads, dim) of q_dtype          */
    int32_t q_dtype;
    int64_t q_batch_stride, q_head_stride;       /* elements                    */
    const void *k_codes, *v_codes;
    int32_t code_bytes;                          /* 1 (uint8) or 2 (u/int16)     */
    int64_t kv_batch_stride, kv_head_stride;     /* codes                       */
    const int32_t *seq_lens;                     /* device, optional            */
    float scale;
    float *out;                                  /* (batch, q_heads, dim) f32   */
    int64_t out_batch_stride, out_head_stride;   /* elements                    */
    int32_t num_splits;                          /* 0 = choose                  */
    int32_t partial_only;
    float *partial_out;
} pkv_attn_args;

/* ---- entry points ------------------------------------------------------ */
PKV_API int pkv_abi_version(void);
PKV_API const char *pkv_strerror(int status);

/* Reads (and optionally clears) the device error word set by a kernel whose
 * bounded wait expired.  Synchronous on the current device.                */
PKV_API int pkv_device_error(int32_t *flag_out, int32_t clear);

/* codes[n, j] for n < N, j < m.  x: (N, dim) rows of x_dtype, row stride
 * x_stride elements.  codes: row stride code_stride codes of code_bytes
 * (1 = uint8, 2 = uint16, 8 = int64).                                     */
PKV_API int pkv_encode(const pkv_codec *c, const void *x, int32_t x_dtype, int64_t n,
               int64_t x_stride, void *codes, int32_t code_bytes,
               int64_t code_stride, void *stream);

/* out[n, :] = dequant(codes[n, :]) @ R, out of out_dtype, row stride
 * out_stride elements.                                                    */
PKV_API int pkv_decode(const pkv_codec *c, const void *codes, int32_t code_bytes,
               int64_t n, int64_t code_stride, void *out, int32_t out_dtype,
               int64_t out_stride, void *stream);

/* KV-cache forms of encode / decode.  The cache holds n_groups (batch x kv
 * head) rows of token slots: slot t of group g at
 * codes + (g * group_stride + t * code_stride) codes.
 * pkv_encode_append encodes x rows (g, i) = x + (g * n_rows + i) * x_stride
 * into slots pos + i of every group -- the device-side append that replaces
 * the torch.cat of RawKVCache.update (cache/raw_cache.py:137-147) and
 * PrismKVCache.update (cache/kv_cache.py:121-131).  pkv_decode_cache decodes
 * slots [pos, pos + n_rows) of every group to out rows g * n_rows + i
 * (RawKVCache.update's backend.decompress, raw_cache.py:150-159).        */
PKV_API int pkv_encode_append(const pkv_codec *c, const void *x, int32_t x_dtype, int64_t n_groups,
                      int64_t n_rows, int64_t x_stride, void *codes, int32_t code_bytes,
                      int64_t group_stride, int64_t code_stride, int64_t pos, void *stream);
PKV_API int pkv_decode_cache(const pkv_codec *c, const void *codes, int32_t code_bytes, int64_t n_groups,
                     int64_t n_rows, int64_t group_stride, int64_t code_stride, int64_t pos,
                     void *out, int32_t out_dtype, int64_t out_stride, void *stream);

/* Bytes of workspace pkv_attn_decode needs for these arguments (0 when one
 * split per KV head suffices).  The workspace must be zeroed once
 * (pkv_workspace_init) before its first use; every call leaves it zeroed. */
PKV_API size_t pkv_attn_workspace_size(const pkv_codec *c, const pkv_attn_args *a);
PKV_API int pkv_workspace_init(void *workspace, size_t bytes, void *stream);
PKV_API int pkv_attn_decode(const pkv_codec *c, const pkv_attn_args *a,
                    void *workspace, size_t workspace_bytes, void *stream);

/* Which kernel and split plan pkv_attn_decode would use for these arguments
 * (introspection for tests and benchmarks; launches nothing; the output
 * pointers of `a` may be null).                                           */
enum { PKV_KERNEL_MHA12 = 1, PKV_KERNEL_POLAR = 2, PKV_KERNEL_LUT = 3, PKV_KERNEL_TC = 4, PKV_KERNEL_MHA8 = 5,
       PKV_KERNEL_MHA12_STREAM = 6, PKV_KERNEL_GQA12 = 7, PKV_KERNEL_GQA12_MMA = 8 };
typedef struct pkv_attn_plan {
    int32_t kernel;            /* PKV_KERNEL_*                                  */
    int32_t num_splits;        /* sequence splits per (batch, kv head)          */
    int32_t tokens_per_split;
    int32_t threads;           /* per CTA                                       */
    int32_t smem_bytes;        /* dynamic shared memory per CTA                 */
    int32_t ctas_per_sm;       /* residency the schedule is planned for         */
    int32_t balanced;          /* 1: every CTA streams an equal share of token
                                  tiles (num_splits = partial slots per row);
                                  0: round-robin over (batch, kv head, split)  */
} pkv_attn_plan;
PKV_API int pkv_attn_describe(const pkv_codec *c, const pkv_attn_args *a, pkv_attn_plan *out);

/* pkv_attn_decode without a caller workspace: the split partials and arrival
 * counters live in one static device array of PKV_NOALLOC_SCRATCH_BYTES
 * (8 MiB) per device, for callers that cannot allocate device memory on the
 * decode path (a C/C++ host without a caching allocator, where cudaMalloc
 * would synchronise the device every step).  It has no counterpart in the
 * reference.  Limits: the partials, batch * q_heads * splits * (dim + 2)
 * floats rounded up to 256 bytes, must fit in 8 MiB - 64 KiB, and the
 * split's arrival counters -- batch * kv_heads, or batch * q_heads when
 * grouped heads of 12-bit codes run one query head per unit -- must not
 * exceed PKV_NOALLOC_MAX_KV_ROWS; otherwise PKV_ERR_SCRATCH_LIMIT and
 * nothing is launched.  Every call
 * looks the array's address up for the current context (cudaGetSymbolAddress,
 * with the device current); the first call that sees an address on a device
 * also zeroes its counter region on `stream` -- make that call before any
 * stream capture.  The counters must be zero when a kernel starts;
 * each call leaves them zero.  The array is shared: calls that overlap in
 * time on one device (other streams, unsynchronised threads) race on it.   */
#define PKV_NOALLOC_SCRATCH_BYTES (8u << 20)
#define PKV_NOALLOC_MAX_KV_ROWS 16384
PKV_API int pkv_attn_decode_noalloc(const pkv_codec *c, const pkv_attn_args *a, void *stream);

/* Merge n_parts partials per row (row r of part p at
 * partials + p*part_stride + r*(dim+2)), normalise, rotate back with R and
 * write out + r*out_row_stride (dim floats).                              */
PKV_API int pkv_lse_combine(const pkv_codec *c, const float *partials, int32_t n_parts,
                    int64_t part_stride, int32_t rows, float *out,
                    int64_t out_row_stride, void *stream);

/* pkv_lse_combine with each part behind its own pointer: `part_ptrs` is a
 * DEVICE array of n_parts pointers; part p of row r is at
 * part_ptrs[p] + part_offset + r*(dim+2).  The pointers may name peer GPUs'
 * buffers mapped over NVLink (split-sequence decode: every rank reads all
 * ranks' partials directly, after a barrier, instead of an all-gather).   */
PKV_API int pkv_lse_combine_gather(const pkv_codec *c, const float *const *part_ptrs, int32_t n_parts,
                           int64_t part_offset, int32_t rows, float *out, int64_t out_row_stride,
                           void *stream);

/* ---- split-sequence decode across GPUs (one process per GPU) ------------ *
 * Each rank holds a contiguous token shard of every (batch, KV head) and runs
 * pkv_attn_decode_xr over it.  The exchange happens inside that one kernel:
 * when a unit's (batch row, its query heads) partial softmax state
 * [m (log2 units), l, o_rot[dim]] is final on a rank, the rank stores it into
 * slot `rank` of EVERY rank's exchange buffer (plain peer stores over NVLink),
 * each value as one 8-byte word (value, flag) whose flag names the call, so
 * no fences or counters order the exchange.  After its last item every CTA
 * of every rank merges its share of the units (unit u on CTA u mod grid):
 * it waits for the flags of all ranks' rows of the unit in its own buffer --
 * bounded by wait_limit_us, measured with the device clock -- merges them
 * (log-sum-exp), applies R once and stores the rank's own output rows.  Every
 * rank computes the same outputs.  The call flag is the rank's call count
 * (kept in the buffer, advanced by the call's last CTA); the partial slots
 * alternate with its parity, so a rank one call ahead cannot overwrite rows a
 * slower rank still reads.  On expiry the device error word is set to 4 (read
 * by pkv_device_error); every rank must then call pkv_xr_reset (after a
 * host-side agreement that the step failed) before the next step.  The
 * buffers are plain cudaMalloc memory (no NVSwitch object) mapped into the
 * peers with CUDA IPC.  The reference has no counterpart: it decodes on one
 * CPU (polar_attention.py:277-309); sharding the sequence is the
 * decomposition of that same softmax.
 *
 * Buffer layout (pkv_xr_layout): partial slots [2][world][rows][dim + 2] of
 * 8-byte (f32 value, u32 flag) words, output rows [rows][dim] f32 (rows =
 * batch * q_heads, row b * q_heads + h), two control words (call count, CTA
 * count); zero when allocated.                                              */
#define PKV_XR_MAX_RANKS 8
typedef struct pkv_exchange {
    int32_t world, rank;
    void *buffers[PKV_XR_MAX_RANKS];   /* every rank's buffer, mapped in this process */
    uint32_t wait_limit_us;            /* bound on the completion wait              */
} pkv_exchange;
typedef struct pkv_xr_layout {
    uint64_t bytes;                    /* buffer size                               */
    uint64_t out_offset;               /* byte offset of the output rows            */
    int32_t rows, units;
} pkv_xr_layout;
PKV_API int pkv_xr_layout_for(const pkv_codec *c, const pkv_attn_args *a, int32_t world, pkv_xr_layout *out);
/* Set-up (not the decode path): allocate a zeroed exchange buffer and export
 * its CUDA IPC handle (64 bytes); open / close a peer's buffer from its
 * handle; free this rank's buffer (after every peer has closed it).          */
PKV_API int pkv_xr_alloc(uint64_t bytes, void **dev_ptr, void *ipc_handle_out);
PKV_API int pkv_xr_open(const void *ipc_handle, void **dev_ptr);
PKV_API int pkv_xr_close(void *peer_ptr);
PKV_API int pkv_xr_free(void *dev_ptr);
/* Zero this rank's buffer, call count included (after an expired wait; every
 * rank, between steps).                                                      */
PKV_API int pkv_xr_reset(const pkv_codec *c, const pkv_attn_args *a, const pkv_exchange *x, void *stream);
/* a->partial_only must be 0 and a->out is unused: outputs land in this rank's
 * buffer at out_offset (every rank merges its own copy).  a->seq_len is this rank's shard length; batch, heads
 * and the plan's unit decomposition must agree across ranks.                  */
PKV_API int pkv_attn_decode_xr(const pkv_codec *c, const pkv_attn_args *a, void *workspace, size_t workspace_bytes,
                               const pkv_exchange *x, void *stream);

/* Scores of prismkv_cuda.polar_attn_fwd: out[b,h,i,j] =
 * scale * <q_rot[b,h,i], dequant(k_codes[b,h,j])> with the uniform polar
 * dequant.  q_params (host): {z_min, delta_z, r_max, delta_r, delta_theta,
 * scale}; bits (host): {bits_z, bits_r, bits_theta}.  q_rot, out fp32
 * contiguous; k_codes contiguous (B, H, Sk, dim/3).                       */
PKV_API int pkv_polar_scores(const float *q_rot, const void *k_codes, int32_t code_bytes,
                     int32_t B, int32_t H, int32_t Sq, int32_t Sk, int32_t dim,
                     const float *q_params, const int32_t *bits, float *out,
                     void *stream);

#ifdef __cplusplus
}
#endif
#endif /* PRISMKV_B200_H */
