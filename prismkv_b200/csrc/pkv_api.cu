// pkv_api.cu -- extern "C" entry points: argument checks, then kernel launch.
//
// Errors are reported as status codes, never by trapping on the device; the
// Python shim turns them into RuntimeError(pkv_strerror(rc)), as the
// reference's TORCH_CHECKs raise (polar_attn_kernel.cu:274-309).

#include <cmath>
#include <cstring>

#include "pkv_common.cuh"

namespace pkv {
int launch_encode(const pkv_codec* c, const void* x, int xdt, int64_t n, int64_t xs, void* codes, int cb,
                  int64_t cs, int64_t group_rows, int64_t group_stride, cudaStream_t st);
int launch_decode(const pkv_codec* c, const void* codes, int cb, int64_t n, int64_t cs, void* out, int odt,
                  int64_t os, int64_t group_rows, int64_t group_stride, cudaStream_t st);
size_t attn_workspace_size(const pkv_codec* c, const pkv_attn_args* a);
void describe_attn(const pkv_codec* c, const pkv_attn_args* a, pkv_attn_plan* out);
bool attn_group_supported(const pkv_codec* c, const pkv_attn_args* a);
int launch_attn(const pkv_codec* c, const pkv_attn_args* a, void* ws, size_t ws_bytes, cudaStream_t st,
                const pkv_exchange* xr = nullptr);
void xr_layout(const pkv_codec* c, const pkv_attn_args* a, int world, pkv_xr_layout* out);
void xr_counter_span(const pkv_codec* c, const pkv_attn_args* a, int world, size_t* off, size_t* len);
int launch_lse_combine(const pkv_codec* c, const float* parts, int n_parts, int64_t part_stride, int rows,
                       float* out, int64_t out_rs, cudaStream_t st);
int launch_lse_combine_gather(const pkv_codec* c, const float* const* part_ptrs, int n_parts, int64_t part_offset,
                              int rows, float* out, int64_t out_rs, cudaStream_t st);
int launch_polar_scores(const float* q, const void* kc, int cb, int B, int H, int Sq, int Sk, int dim,
                        const float* qp, const int32_t* bits, float* out, cudaStream_t st);
}  // namespace pkv

namespace {

bool valid_dtype(int dt) { return dt == PKV_F32 || dt == PKV_BF16 || dt == PKV_F16; }

int check_codec(const pkv_codec* c, bool need_encode, bool need_decode) {
    if (!c) return PKV_ERR_INVALID;
    if (c->dim <= 0 || c->dim % 3 != 0) return PKV_ERR_INVALID;
    if (c->dim > 192) return PKV_ERR_UNSUPPORTED;
    const int b[3] = {c->bits_z, c->bits_r, c->bits_theta};
    for (int i = 0; i < 3; ++i)
        if (b[i] < 1 || b[i] > PKV_MAX_BITS) return PKV_ERR_INVALID;
    if (b[0] + b[1] + b[2] > PKV_MAX_TOTAL_BITS) return PKV_ERR_INVALID;
    if (c->xy_mode != 0 && c->xy_mode != 1) return PKV_ERR_INVALID;
    if (!c->R) return PKV_ERR_INVALID;
    if (need_encode) {
        if (!c->z_thr) return PKV_ERR_INVALID;
        if (c->xy_mode == 0 && (!c->r2_thr || !c->th_thr)) return PKV_ERR_INVALID;
        if (c->xy_mode == 1 && !c->codebook) return PKV_ERR_INVALID;
        if (c->z_nan_bin < 0 || c->z_nan_bin >= (1 << c->bits_z)) return PKV_ERR_INVALID;
    }
    if (need_decode && (!c->dec_z || !c->dec_xy)) return PKV_ERR_INVALID;
    return PKV_OK;
}

int code_bits_fit(const pkv_codec* c, int code_bytes) {
    const int total = c->bits_z + c->bits_r + c->bits_theta;
    if (code_bytes == 1) return total <= 8;
    if (code_bytes == 2 || code_bytes == 8) return 1;
    return 0;
}

}  // namespace

extern "C" {

int pkv_abi_version(void) { return PKV_ABI_VERSION; }

const char* pkv_strerror(int status) {
    switch (status) {
        case PKV_OK: return "ok";
        case PKV_ERR_INVALID: return "invalid argument (null pointer, shape, dtype or bit widths)";
        case PKV_ERR_UNSUPPORTED: return "unsupported configuration for this library";
        case PKV_ERR_ALIGNMENT: return "misaligned pointer or stride";
        case PKV_ERR_WORKSPACE: return "workspace missing or too small";
        case PKV_ERR_CUDA: return "CUDA runtime error";
        case PKV_ERR_DEVICE: return "device-side error flag set (a bounded wait expired)";
        case PKV_ERR_SCRATCH_LIMIT:
            return "arguments need more split scratch than the static array of pkv_attn_decode_noalloc holds "
                   "(8 MiB - 64 KiB of partials, 16384 split counters); use pkv_attn_decode with a workspace";
    }
    return "unknown status";
}

int pkv_device_error(int32_t* flag_out, int32_t clear) {
    if (!flag_out) return PKV_ERR_INVALID;
    if (cudaMemcpyFromSymbol(flag_out, pkv::g_device_error, sizeof(int32_t)) != cudaSuccess) return PKV_ERR_CUDA;
    if (clear) {
        const int32_t zero = 0;
        if (cudaMemcpyToSymbol(pkv::g_device_error, &zero, sizeof(int32_t)) != cudaSuccess) return PKV_ERR_CUDA;
    }
    return PKV_OK;
}

int pkv_encode(const pkv_codec* c, const void* x, int32_t x_dtype, int64_t n, int64_t x_stride, void* codes,
               int32_t code_bytes, int64_t code_stride, void* stream) {
    int rc = check_codec(c, true, false);
    if (rc) return rc;
    if (n < 0 || !valid_dtype(x_dtype)) return PKV_ERR_INVALID;
    if (!code_bits_fit(c, code_bytes)) return PKV_ERR_INVALID;
    if (n == 0) return PKV_OK;
    if (!x || !codes || x_stride < c->dim || code_stride < c->dim / 3) return PKV_ERR_INVALID;
    return pkv::launch_encode(c, x, x_dtype, n, x_stride, codes, code_bytes, code_stride, 0, 0,
                              static_cast<cudaStream_t>(stream));
}

int pkv_decode(const pkv_codec* c, const void* codes, int32_t code_bytes, int64_t n, int64_t code_stride,
               void* out, int32_t out_dtype, int64_t out_stride, void* stream) {
    int rc = check_codec(c, false, true);
    if (rc) return rc;
    if (n < 0 || !valid_dtype(out_dtype)) return PKV_ERR_INVALID;
    if (!code_bits_fit(c, code_bytes)) return PKV_ERR_INVALID;
    if (n == 0) return PKV_OK;
    if (!codes || !out || out_stride < c->dim || code_stride < c->dim / 3) return PKV_ERR_INVALID;
    return pkv::launch_decode(c, codes, code_bytes, n, code_stride, out, out_dtype, out_stride, 0, 0,
                              static_cast<cudaStream_t>(stream));
}

// The code side of a KV cache: n_groups (batch x head) rows of `capacity`
// token slots, group_stride codes apart.  Rows [pos, pos + n_rows) of each group.
static int check_cache_rows(const pkv_codec* c, int64_t n_groups, int64_t n_rows, int64_t group_stride,
                            int64_t code_stride, int64_t pos) {
    if (n_groups < 0 || n_rows < 0 || pos < 0) return PKV_ERR_INVALID;
    if (code_stride < c->dim / 3) return PKV_ERR_INVALID;
    if (n_groups > 1 && group_stride < (pos + n_rows) * code_stride) return PKV_ERR_INVALID;
    return PKV_OK;
}

int pkv_encode_append(const pkv_codec* c, const void* x, int32_t x_dtype, int64_t n_groups, int64_t n_rows,
                      int64_t x_stride, void* codes, int32_t code_bytes, int64_t group_stride,
                      int64_t code_stride, int64_t pos, void* stream) {
    int rc = check_codec(c, true, false);
    if (rc) return rc;
    if (!valid_dtype(x_dtype) || !code_bits_fit(c, code_bytes)) return PKV_ERR_INVALID;
    rc = check_cache_rows(c, n_groups, n_rows, group_stride, code_stride, pos);
    if (rc) return rc;
    if (n_groups * n_rows == 0) return PKV_OK;
    if (!x || !codes || x_stride < c->dim) return PKV_ERR_INVALID;
    uint8_t* first = static_cast<uint8_t*>(codes) + pos * code_stride * code_bytes;
    return pkv::launch_encode(c, x, x_dtype, n_groups * n_rows, x_stride, first, code_bytes, code_stride, n_rows,
                              group_stride, static_cast<cudaStream_t>(stream));
}

int pkv_decode_cache(const pkv_codec* c, const void* codes, int32_t code_bytes, int64_t n_groups, int64_t n_rows,
                     int64_t group_stride, int64_t code_stride, int64_t pos, void* out, int32_t out_dtype,
                     int64_t out_stride, void* stream) {
    int rc = check_codec(c, false, true);
    if (rc) return rc;
    if (!valid_dtype(out_dtype) || !code_bits_fit(c, code_bytes)) return PKV_ERR_INVALID;
    rc = check_cache_rows(c, n_groups, n_rows, group_stride, code_stride, pos);
    if (rc) return rc;
    if (n_groups * n_rows == 0) return PKV_OK;
    if (!codes || !out || out_stride < c->dim) return PKV_ERR_INVALID;
    const uint8_t* first = static_cast<const uint8_t*>(codes) + pos * code_stride * code_bytes;
    return pkv::launch_decode(c, first, code_bytes, n_groups * n_rows, code_stride, out, out_dtype, out_stride,
                              n_rows, group_stride, static_cast<cudaStream_t>(stream));
}

static int check_attn(const pkv_codec* c, const pkv_attn_args* a, bool need_out = true) {
    int rc = check_codec(c, false, true);
    if (rc) return rc;
    if (!a) return PKV_ERR_INVALID;
    if (a->batch < 0 || a->q_heads < 0 || a->kv_heads < 0 || a->seq_len < 0) return PKV_ERR_INVALID;
    if (a->kv_heads == 0 || a->q_heads == 0 || a->q_heads % a->kv_heads != 0) return PKV_ERR_INVALID;
    if (a->q_heads / a->kv_heads > 16) return PKV_ERR_UNSUPPORTED;   // > 8 only where the plan allows (below)
    if (a->code_bytes != 1 && a->code_bytes != 2) return PKV_ERR_INVALID;
    if (!code_bits_fit(c, a->code_bytes)) return PKV_ERR_INVALID;
    if (c->bits_z + c->bits_r + c->bits_theta > 12) return PKV_ERR_UNSUPPORTED;
    if (!valid_dtype(a->q_dtype)) return PKV_ERR_INVALID;
    if (!(std::isfinite(a->scale))) return PKV_ERR_INVALID;
    if (a->num_splits < 0) return PKV_ERR_INVALID;
    if (a->batch == 0) return PKV_OK;
    if (!a->q || (a->seq_len > 0 && (!a->k_codes || !a->v_codes))) return PKV_ERR_INVALID;
    if (need_out && (a->partial_only ? !a->partial_out : !a->out)) return PKV_ERR_INVALID;
    const int64_t m = c->dim / 3;
    if (a->kv_head_stride < (int64_t)a->seq_len * m || a->kv_batch_stride < 0) return PKV_ERR_INVALID;
    return PKV_OK;
}

size_t pkv_attn_workspace_size(const pkv_codec* c, const pkv_attn_args* a) {
    if (check_attn(c, a) != PKV_OK || a->batch == 0 || !pkv::attn_group_supported(c, a)) return 0;
    return pkv::attn_workspace_size(c, a);
}

int pkv_attn_describe(const pkv_codec* c, const pkv_attn_args* a, pkv_attn_plan* out) {
    if (!out) return PKV_ERR_INVALID;
    const int rc = check_attn(c, a, false);     // output pointers are not needed to plan
    if (rc) return rc;
    if (!pkv::attn_group_supported(c, a)) return PKV_ERR_UNSUPPORTED;
    pkv::describe_attn(c, a, out);
    return PKV_OK;
}

int pkv_workspace_init(void* workspace, size_t bytes, void* stream) {
    if (bytes == 0) return PKV_OK;
    if (!workspace) return PKV_ERR_INVALID;
    return cudaMemsetAsync(workspace, 0, bytes, static_cast<cudaStream_t>(stream)) == cudaSuccess ? PKV_OK
                                                                                              : PKV_ERR_CUDA;
}

int pkv_attn_decode(const pkv_codec* c, const pkv_attn_args* a, void* workspace, size_t workspace_bytes,
                    void* stream) {
    int rc = check_attn(c, a);
    if (rc) return rc;
    if (a->batch == 0) return PKV_OK;
    return pkv::launch_attn(c, a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

// ---- split-sequence exchange ----------------------------------------------
static int check_xr(const pkv_exchange* x) {
    if (!x || x->world < 1 || x->world > PKV_XR_MAX_RANKS || x->rank < 0 || x->rank >= x->world) return PKV_ERR_INVALID;
    for (int s = 0; s < x->world; ++s)
        if (!x->buffers[s] || reinterpret_cast<uintptr_t>(x->buffers[s]) % 256 != 0) return PKV_ERR_INVALID;
    return PKV_OK;
}

int pkv_xr_layout_for(const pkv_codec* c, const pkv_attn_args* a, int32_t world, pkv_xr_layout* out) {
    if (!out || world < 1 || world > PKV_XR_MAX_RANKS) return PKV_ERR_INVALID;
    const int rc = check_attn(c, a, false);
    if (rc) return rc;
    if (!pkv::attn_group_supported(c, a)) return PKV_ERR_UNSUPPORTED;
    pkv::xr_layout(c, a, world, out);
    return PKV_OK;
}

int pkv_xr_alloc(uint64_t bytes, void** dev_ptr, void* ipc_handle_out) {
    if (!dev_ptr || !ipc_handle_out || bytes == 0) return PKV_ERR_INVALID;
    void* ptr = nullptr;
    if (cudaMalloc(&ptr, bytes) != cudaSuccess) return PKV_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaMemset(ptr, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) {
        cudaFree(ptr);
        return PKV_ERR_CUDA;
    }
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    memcpy(ipc_handle_out, &h, sizeof(h));
    *dev_ptr = ptr;
    return PKV_OK;
}

int pkv_xr_open(const void* ipc_handle, void** dev_ptr) {
    if (!ipc_handle || !dev_ptr) return PKV_ERR_INVALID;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    return cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? PKV_OK : PKV_ERR_CUDA;
}

int pkv_xr_close(void* peer_ptr) {
    if (!peer_ptr) return PKV_ERR_INVALID;
    return cudaIpcCloseMemHandle(peer_ptr) == cudaSuccess ? PKV_OK : PKV_ERR_CUDA;
}

int pkv_xr_free(void* dev_ptr) {
    if (!dev_ptr) return PKV_ERR_INVALID;
    return cudaFree(dev_ptr) == cudaSuccess ? PKV_OK : PKV_ERR_CUDA;
}

int pkv_xr_reset(const pkv_codec* c, const pkv_attn_args* a, const pkv_exchange* x, void* stream) {
    int rc = check_xr(x);
    if (rc) return rc;
    rc = check_attn(c, a, false);
    if (rc) return rc;
    size_t off = 0, len = 0;
    pkv::xr_counter_span(c, a, x->world, &off, &len);
    return cudaMemsetAsync(static_cast<uint8_t*>(x->buffers[x->rank]) + off, 0, len,
                           static_cast<cudaStream_t>(stream)) == cudaSuccess ? PKV_OK : PKV_ERR_CUDA;
}

int pkv_attn_decode_xr(const pkv_codec* c, const pkv_attn_args* a, void* workspace, size_t workspace_bytes,
                       const pkv_exchange* x, void* stream) {
    int rc = check_xr(x);
    if (rc) return rc;
    if (a && a->partial_only) return PKV_ERR_INVALID;
    rc = check_attn(c, a, false);
    if (rc) return rc;
    if (a->batch == 0) return PKV_OK;
    if (!pkv::attn_group_supported(c, a)) return PKV_ERR_UNSUPPORTED;
    return pkv::launch_attn(c, a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), x);
}

int pkv_lse_combine(const pkv_codec* c, const float* partials, int32_t n_parts, int64_t part_stride, int32_t rows,
                    float* out, int64_t out_row_stride, void* stream) {
    if (!c || c->dim <= 0 || c->dim % 3 != 0 || !c->R) return PKV_ERR_INVALID;
    if (c->dim > 192) return PKV_ERR_UNSUPPORTED;
    if (n_parts < 1 || rows < 0) return PKV_ERR_INVALID;
    if (rows == 0) return PKV_OK;
    if (!partials || !out || out_row_stride < c->dim) return PKV_ERR_INVALID;
    if (n_parts > 1 && part_stride < (int64_t)rows * (c->dim + 2)) return PKV_ERR_INVALID;
    return pkv::launch_lse_combine(c, partials, n_parts, part_stride, rows, out, out_row_stride,
                                   static_cast<cudaStream_t>(stream));
}

int pkv_lse_combine_gather(const pkv_codec* c, const float* const* part_ptrs, int32_t n_parts, int64_t part_offset,
                           int32_t rows, float* out, int64_t out_row_stride, void* stream) {
    if (!c || c->dim <= 0 || c->dim % 3 != 0 || !c->R) return PKV_ERR_INVALID;
    if (c->dim > 192) return PKV_ERR_UNSUPPORTED;
    if (n_parts < 1 || rows < 0 || part_offset < 0) return PKV_ERR_INVALID;
    if (rows == 0) return PKV_OK;
    if (!part_ptrs || !out || out_row_stride < c->dim) return PKV_ERR_INVALID;
    return pkv::launch_lse_combine_gather(c, part_ptrs, n_parts, part_offset, rows, out, out_row_stride,
                                          static_cast<cudaStream_t>(stream));
}

int pkv_polar_scores(const float* q_rot, const void* k_codes, int32_t code_bytes, int32_t B, int32_t H, int32_t Sq,
                     int32_t Sk, int32_t dim, const float* q_params, const int32_t* bits, float* out,
                     void* stream) {
    if (!q_params || !bits) return PKV_ERR_INVALID;
    if (B < 0 || H < 0 || Sq < 0 || Sk < 0 || dim <= 0 || dim % 3 != 0) return PKV_ERR_INVALID;
    if (dim > 192) return PKV_ERR_UNSUPPORTED;
    for (int i = 0; i < 3; ++i)
        if (bits[i] < 1 || bits[i] > PKV_MAX_BITS) return PKV_ERR_INVALID;
    if (bits[0] + bits[1] + bits[2] > PKV_MAX_TOTAL_BITS) return PKV_ERR_INVALID;
    if (code_bytes != 1 && code_bytes != 2) return PKV_ERR_INVALID;
    if (code_bytes == 1 && bits[0] + bits[1] + bits[2] > 8) return PKV_ERR_INVALID;
    if ((int64_t)B * H * Sq * Sk == 0) return PKV_OK;
    if (!q_rot || !k_codes || !out) return PKV_ERR_INVALID;
    return pkv::launch_polar_scores(q_rot, k_codes, code_bytes, B, H, Sq, Sk, dim, q_params, bits, out,
                                    static_cast<cudaStream_t>(stream));
}

}  // extern "C"
