// capi.cu -- the extern "C" entry points declared in include/densecore_sdpa.h.
//
// Validation follows DenseCore's pyo3 boundary (src/lib.rs): attention_dims (:555-580)
// requires 4-D tensors, k and v of equal batch/length, equal head dim for q and k, and
// H % Hkv == 0; attention_mask (:594-607) checks the mask against (B, H, L, S) -- here a
// broadcastable strided mask is accepted instead of a materialised one; the backward checks
// grad_out/out against q's shape and lse against (B, H, L) (:658-662). Shape errors return
// DC_ERR_VALUE (the reference raises ValueError), kernel failures DC_ERR_RUNTIME or
// DC_ERR_CUDA (RuntimeError).
#include <cuda_runtime.h>
#include <math.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace dc {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string &msg) { g_last_error = msg; }

std::string last_error() { return g_last_error; }

int fail(int status, const std::string &msg) {
    g_last_error = msg;
    return status;
}

int cuda_fail(cudaError_t err, const char *what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(err);
    return DC_ERR_CUDA;
}

int check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DC_OK : cuda_fail(e, what);
}

namespace {

std::string shape_str(const dc_tensor_t *t) {
    std::string s = "(";
    for (int i = 0; i < t->ndim; i++) s += (i ? ", " : "") + std::to_string(t->sizes[i]);
    return s + ")";
}

bool is_f32(const dc_tensor_t *t, int ndim) {
    return t && t->dtype == DC_F32 && t->ndim == ndim;
}

bool sizes_are(const dc_tensor_t *t, std::initializer_list<int64_t> want) {
    int i = 0;
    for (int64_t w : want) {
        if (i >= t->ndim || t->sizes[i] != w) return false;
        i++;
    }
    return i == t->ndim;
}

void copy_strides(const dc_tensor_t *t, int64_t *dst, int n) {
    for (int i = 0; i < n; i++) dst[i] = t->strides[i];
}

// attention_dims (src/lib.rs:555-580), generalised to Ev != E.
int fill_problem(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *v, int causal,
                 int has_scale, double scale, AttnProblem &p) {
    if (!q || !k || !v) return fail(DC_ERR_VALUE, "flash attention: q, k and v are required");
    if (!is_f32(q, 4) || !is_f32(k, 4) || !is_f32(v, 4))
        return fail(DC_ERR_VALUE, "flash attention takes (B, H, L, E) float32 tensors");
    const int64_t *qs = q->sizes, *ks = k->sizes, *vs = v->sizes;
    bool ok = ks[0] == qs[0] && vs[0] == ks[0] && ks[1] == vs[1] && ks[2] == vs[2] &&
              ks[3] == qs[3] && ks[1] > 0 && qs[1] % ks[1] == 0;
    for (int i = 0; i < 4; i++) ok = ok && qs[i] >= 0 && ks[i] >= 0 && vs[i] >= 0;
    if (!ok)
        return fail(DC_ERR_VALUE, "flash attention q/k/v shapes do not match: q " + shape_str(q) +
                                      ", k " + shape_str(k) + ", v " + shape_str(v));
    p = AttnProblem{};
    p.q = static_cast<const float *>(q->data);
    p.k = static_cast<const float *>(k->data);
    p.v = static_cast<const float *>(v->data);
    p.B = qs[0];
    p.H = qs[1];
    p.Hkv = ks[1];
    p.L = qs[2];
    p.S = ks[2];
    p.E = qs[3];
    p.Ev = vs[3];
    copy_strides(q, p.qs, 4);
    copy_strides(k, p.ks, 4);
    copy_strides(v, p.vs, 4);
    p.causal = causal ? 1 : 0;
    // scale_factor (torch_attention.rs:37-40): computed in double, stored as float.
    p.scale = has_scale ? (float)scale : (float)(1.0 / sqrt((double)p.E));
    p.group = (int)(p.H / p.Hkv);
    if (p.H > 65535 || p.B > 65535)
        return fail(DC_ERR_UNSUPPORTED, "batch and head counts above 65535 are not supported");
    return DC_OK;
}

// attention_mask (src/lib.rs:594-607), generalised: 2-4 dims broadcastable to (B,H,L,S).
int fill_mask(const dc_tensor_t *mask, AttnProblem &p) {
    p.mask = nullptr;
    p.mask_kind = MASK_NONE;
    for (int i = 0; i < 4; i++) p.ms[i] = 0;
    if (!mask) return DC_OK;
    if (mask->ndim < 2 || mask->ndim > 4 || (mask->dtype != DC_F32 && mask->dtype != DC_BOOL))
        return fail(DC_ERR_VALUE, "flash attention mask must be a float32 or bool tensor of 2 to 4 dims");
    const int64_t want[4] = {p.B, p.H, p.L, p.S};
    const int pad = 4 - mask->ndim;
    for (int i = 0; i < 4; i++) {
        if (i < pad) continue;
        const int64_t sz = mask->sizes[i - pad];
        if (sz == want[i]) {
            p.ms[i] = want[i] == 1 ? 0 : mask->strides[i - pad];
        } else if (sz == 1) {
            p.ms[i] = 0;
        } else {
            return fail(DC_ERR_VALUE, "flash attention mask " + shape_str(mask) +
                                          " does not broadcast to (B, H, L, S)");
        }
    }
    p.mask = mask->data;
    p.mask_kind = mask->dtype == DC_F32 ? MASK_FLOAT : MASK_BOOL;
    return DC_OK;
}

int check_out(const dc_tensor_t *out, const dc_tensor_t *lse, const AttnProblem &p) {
    if (!is_f32(out, 4) || !sizes_are(out, {p.B, p.H, p.L, p.Ev}))
        return fail(DC_ERR_VALUE, "flash attention output must be float32 (B, H, L, Ev)");
    if (!is_f32(lse, 3) || !sizes_are(lse, {p.B, p.H, p.L}))
        return fail(DC_ERR_VALUE, "flash attention logsumexp must be float32 (B, H, L)");
    return DC_OK;
}

int check_precision(int precision) {
    if (precision < DC_PREC_3XTF32 || precision > DC_PREC_FP32)
        return fail(DC_ERR_VALUE, "unknown precision mode " + std::to_string(precision));
    return DC_OK;
}

int device_ok() {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_fail(e, "no CUDA device");
    if (n == 0) return fail(DC_ERR_CUDA, "no CUDA device");
    return DC_OK;
}

struct ScopedWorkspace {
    void *ptr = nullptr;
    bool owned = false;
    cudaStream_t stream = nullptr;
    ~ScopedWorkspace() {
        if (owned && ptr) cudaFreeAsync(ptr, stream);
    }
    int get(void *given, size_t given_bytes, size_t need, cudaStream_t s, const char *what) {
        stream = s;
        if (need == 0) return DC_OK;
        if (given) {
            if (given_bytes < need)
                return fail(DC_ERR_VALUE, std::string(what) + ": workspace of " +
                                              std::to_string(given_bytes) + " bytes, " +
                                              std::to_string(need) + " needed");
            ptr = given;
            return DC_OK;
        }
        cudaError_t e = cudaMallocAsync(&ptr, need, s);
        if (e != cudaSuccess) return cuda_fail(e, what);
        owned = true;
        return DC_OK;
    }
};

int pick_forward_path(const AttnProblem &p, int precision) {
    if (p.L == 1 && decode_supported(p)) return 2;
    if (precision != DC_PREC_FP32 && tc_forward_supported(p)) return 1;
    return 0;
}

}  // namespace

// Scratch of dc_sdpa_decode_noalloc: the table of split partials (Ev accumulators, the running
// max and the running sum per split) lives in this fixed device array instead of caller or
// stream-ordered memory. Nothing in it has to start at zero: the split kernel writes every
// slot of the table before the combine kernel reads it, so the array's contents at module
// load are never used.
static __device__ __align__(256) float g_decode_scratch[DC_DECODE_NOALLOC_SCRATCH_BYTES / sizeof(float)];

namespace {

constexpr int kScratchDevices = 64;
std::mutex g_scratch_mu;
void *g_scratch_addr[kScratchDevices];

// Device address of g_decode_scratch on the current device. The lookup runs once per device,
// with that device current (it may load the library's module there), and is cached.
int decode_scratch(void **ptr) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "decode scratch: current device");
    if (dev < 0 || dev >= kScratchDevices)
        return fail(DC_ERR_UNSUPPORTED, "decode scratch: device ordinal " + std::to_string(dev) +
                                            " is above " + std::to_string(kScratchDevices - 1));
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void *addr = nullptr;
        e = cudaGetSymbolAddress(&addr, g_decode_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "decode scratch: cudaGetSymbolAddress");
        g_scratch_addr[dev] = addr;
    }
    *ptr = g_scratch_addr[dev];
    return DC_OK;
}

}  // namespace
}  // namespace dc

using namespace dc;

extern "C" {

const char *dc_last_error(void) { return g_last_error.c_str(); }

int dc_abi_version(void) { return DC_SDPA_ABI_VERSION; }

int dc_device_status(int reset) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cuda_fail(e, "device status");
        return -1;
    }
    return device_error(reset);
}

int dc_sdpa_fwd_path(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *v,
                     const dc_tensor_t *mask, int causal, int precision) {
    AttnProblem p;
    if (fill_problem(q, k, v, causal, 0, 0.0, p) || fill_mask(mask, p)) return -1;
    return pick_forward_path(p, precision);
}

// Dropout arguments shared by the *_dropout entry points: the keep bits of B*H*L*S elements.
static int set_keep(AttnProblem &p, const uint32_t *keep_bits, float keep_scale) {
    if (p.B * p.H * p.L * p.S > 0 && !keep_bits)
        return fail(DC_ERR_VALUE, "dropout: keep_bits must not be null");
    if ((reinterpret_cast<uintptr_t>(keep_bits) & 3u) != 0)
        return fail(DC_ERR_VALUE, "dropout: keep_bits must be 4-byte aligned");
    p.keep = keep_bits;
    p.keep_scale = keep_scale;
    return DC_OK;
}

static int sdpa_fwd_impl(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *v,
                         const dc_tensor_t *mask, int causal, int has_scale, double scale, int precision,
                         const uint32_t *keep_bits, float keep_scale, bool dropout, dc_tensor_t *out,
                         dc_tensor_t *lse, void *stream) {
    AttnProblem p;
    int st = fill_problem(q, k, v, causal, has_scale, scale, p);
    if (!st) st = fill_mask(mask, p);
    if (!st) st = check_out(out, lse, p);
    if (!st) st = check_precision(precision);
    if (!st && dropout) st = set_keep(p, keep_bits, keep_scale);
    if (st) return st;
    p.out = static_cast<float *>(out->data);
    p.lse = static_cast<float *>(lse->data);
    copy_strides(out, p.os, 4);
    copy_strides(lse, p.ls, 3);
    if (p.B == 0 || p.H == 0 || p.L == 0) return DC_OK;
    if ((st = device_ok())) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int path = pick_forward_path(p, precision);
    // With dropout the tensor-core kernels apply the keep bits; the decode and CUDA-core
    // shapes take the CUDA-core kernel, which applies them too.
    if (dropout && path != 1) return simt_forward(p, s);
    switch (path) {
        case 2: {
            const int splits = decode_pick_splits(p);
            ScopedWorkspace ws;
            if ((st = ws.get(nullptr, 0, decode_workspace_bytes(p.B, p.H, p.Ev, splits), s,
                             "decode workspace")))
                return st;
            return decode_forward(p, splits, ws.ptr, s);
        }
        case 1:
            return tc_forward(p, precision, s);
        default:
            return simt_forward(p, s);
    }
}

int dc_sdpa_fwd(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *v,
                const dc_tensor_t *mask, int causal, int has_scale, double scale, int precision,
                dc_tensor_t *out, dc_tensor_t *lse, void *stream) {
    return sdpa_fwd_impl(q, k, v, mask, causal, has_scale, scale, precision, nullptr, 0.0f, false, out, lse,
                         stream);
}

int dc_sdpa_fwd_dropout(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *v,
                        const dc_tensor_t *mask, int causal, int has_scale, double scale, int precision,
                        const uint32_t *keep_bits, float keep_scale, dc_tensor_t *out, dc_tensor_t *lse,
                        void *stream) {
    return sdpa_fwd_impl(q, k, v, mask, causal, has_scale, scale, precision, keep_bits, keep_scale, true, out,
                         lse, stream);
}

size_t dc_sdpa_bwd_workspace_size(int64_t batch, int64_t heads, int64_t q_len) {
    const size_t n = (size_t)(batch > 0 ? batch : 0) * (heads > 0 ? heads : 0) *
                     (q_len > 0 ? q_len : 0);
    return ((n * sizeof(float) + 255) / 256) * 256;
}

static int sdpa_bwd_impl(const dc_tensor_t *grad_out, const dc_tensor_t *q, const dc_tensor_t *k,
                         const dc_tensor_t *v, const dc_tensor_t *out, const dc_tensor_t *lse,
                         const dc_tensor_t *mask, int causal, int has_scale, double scale, int precision,
                         const uint32_t *keep_bits, float keep_scale, bool dropout, dc_tensor_t *grad_q,
                         dc_tensor_t *grad_k, dc_tensor_t *grad_v, void *workspace, size_t workspace_bytes,
                         void *stream) {
    AttnProblem p;
    int st = fill_problem(q, k, v, causal, has_scale, scale, p);
    if (!st) st = fill_mask(mask, p);
    if (!st) st = check_precision(precision);
    if (!st && dropout) st = set_keep(p, keep_bits, keep_scale);
    if (st) return st;
    // src/lib.rs:658-662: grad and out shaped like the output, lse (B, H, L).
    if (!is_f32(grad_out, 4) || !sizes_are(grad_out, {p.B, p.H, p.L, p.Ev}) || !is_f32(out, 4) ||
        !sizes_are(out, {p.B, p.H, p.L, p.Ev}) || !is_f32(lse, 3) ||
        !sizes_are(lse, {p.B, p.H, p.L}))
        return fail(DC_ERR_VALUE, "flash attention backward shapes do not match");
    if (!is_f32(grad_q, 4) || !sizes_are(grad_q, {p.B, p.H, p.L, p.E}) || !is_f32(grad_k, 4) ||
        !sizes_are(grad_k, {p.B, p.Hkv, p.S, p.E}) || !is_f32(grad_v, 4) ||
        !sizes_are(grad_v, {p.B, p.Hkv, p.S, p.Ev}))
        return fail(DC_ERR_VALUE, "flash attention gradient outputs must match q, k and v");
    p.out = static_cast<float *>(out->data);
    p.lse = static_cast<float *>(lse->data);
    copy_strides(out, p.os, 4);
    copy_strides(lse, p.ls, 3);
    AttnGrads g{};
    g.dout = static_cast<const float *>(grad_out->data);
    g.dq = static_cast<float *>(grad_q->data);
    g.dk = static_cast<float *>(grad_k->data);
    g.dv = static_cast<float *>(grad_v->data);
    copy_strides(grad_out, g.dos, 4);
    copy_strides(grad_q, g.dqs, 4);
    copy_strides(grad_k, g.dks, 4);
    copy_strides(grad_v, g.dvs, 4);
    if (p.B == 0 || p.Hkv == 0) return DC_OK;
    if ((st = device_ok())) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ScopedWorkspace ws;
    if ((st = ws.get(workspace, workspace_bytes, dc_sdpa_bwd_workspace_size(p.B, p.H, p.L), s,
                     "backward workspace")))
        return st;
    g.delta = static_cast<float *>(ws.ptr);
    // The tensor-core backward computes delta in its own pre-pass.
    if (precision != DC_PREC_FP32 && tc_backward_supported(p, g)) return tc_backward(p, g, precision, s);
    if (p.L > 0 && (st = bwd_delta(p, g, s))) return st;
    return simt_backward(p, g, s);
}

int dc_sdpa_bwd(const dc_tensor_t *grad_out, const dc_tensor_t *q, const dc_tensor_t *k,
                const dc_tensor_t *v, const dc_tensor_t *out, const dc_tensor_t *lse,
                const dc_tensor_t *mask, int causal, int has_scale, double scale, int precision,
                dc_tensor_t *grad_q, dc_tensor_t *grad_k, dc_tensor_t *grad_v, void *workspace,
                size_t workspace_bytes, void *stream) {
    return sdpa_bwd_impl(grad_out, q, k, v, out, lse, mask, causal, has_scale, scale, precision, nullptr, 0.0f,
                         false, grad_q, grad_k, grad_v, workspace, workspace_bytes, stream);
}

int dc_sdpa_bwd_dropout(const dc_tensor_t *grad_out, const dc_tensor_t *q, const dc_tensor_t *k,
                        const dc_tensor_t *v, const dc_tensor_t *out, const dc_tensor_t *lse,
                        const dc_tensor_t *mask, int causal, int has_scale, double scale, int precision,
                        const uint32_t *keep_bits, float keep_scale, dc_tensor_t *grad_q, dc_tensor_t *grad_k,
                        dc_tensor_t *grad_v, void *workspace, size_t workspace_bytes, void *stream) {
    return sdpa_bwd_impl(grad_out, q, k, v, out, lse, mask, causal, has_scale, scale, precision, keep_bits,
                         keep_scale, true, grad_q, grad_k, grad_v, workspace, workspace_bytes, stream);
}

int dc_dropout_keep_bits(const uint32_t *state_in, uint32_t *state_out, int64_t n, double keep_prob,
                         uint32_t *bits, void *stream) {
    if (n > 0) {
        int st = device_ok();
        if (st) return st;
    }
    return keep_bits(state_in, state_out, n, keep_prob, bits, static_cast<cudaStream_t>(stream));
}

int dc_rng_skip(const uint32_t *state_in, uint64_t outputs, uint32_t *state_out) {
    return rng_skip(state_in, outputs, state_out);
}

size_t dc_sdpa_decode_workspace_size(int64_t batch, int64_t heads, int64_t head_dim_v,
                                     int num_splits) {
    if (batch <= 0 || heads <= 0 || head_dim_v <= 0 || num_splits <= 0) return 0;
    return decode_workspace_bytes(batch, heads, head_dim_v, num_splits);
}

int dc_sdpa_decode_default_splits(int64_t batch, int64_t heads, int64_t kv_len) {
    AttnProblem p{};
    p.B = batch;
    p.H = heads;
    p.S = kv_len;
    return decode_pick_splits(p);
}

int dc_sdpa_decode(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *v,
                   const dc_tensor_t *mask, int has_scale, double scale, int num_splits,
                   dc_tensor_t *out, dc_tensor_t *lse, void *workspace, size_t workspace_bytes,
                   void *stream) {
    AttnProblem p;
    int st = fill_problem(q, k, v, 0, has_scale, scale, p);
    if (!st) st = fill_mask(mask, p);
    if (!st) st = check_out(out, lse, p);
    if (st) return st;
    if (p.L != 1) return fail(DC_ERR_VALUE, "decode takes a query length of 1");
    p.out = static_cast<float *>(out->data);
    p.lse = static_cast<float *>(lse->data);
    copy_strides(out, p.os, 4);
    copy_strides(lse, p.ls, 3);
    if (!decode_supported(p))
        return fail(DC_ERR_UNSUPPORTED,
                    "decode needs head dim 64 or 128, E == Ev, unit-stride rows on 16-byte "
                    "boundaries; use dc_sdpa_fwd");
    if (p.B == 0 || p.H == 0) return DC_OK;
    if ((st = device_ok())) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int splits = num_splits > 0 ? (num_splits > 1024 ? 1024 : num_splits) : decode_pick_splits(p);
    ScopedWorkspace ws;
    if ((st = ws.get(workspace, workspace_bytes, decode_workspace_bytes(p.B, p.H, p.Ev, splits), s,
                     "decode workspace")))
        return st;
    return decode_forward(p, splits, ws.ptr, s);
}

// The split-KV decode of dc_sdpa_decode with its partials in g_decode_scratch. It exists for
// callers that must not have the library allocate: a serving loop that has reserved the
// device's free memory for its KV cache up front (a hidden cudaMallocAsync would then fail or
// eat into the cache), and hosts reaching the library through a plain C FFI that own no
// allocator and cannot hand over a workspace. Everything else matches dc_sdpa_decode.
int dc_sdpa_decode_noalloc(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *v,
                           const dc_tensor_t *mask, int has_scale, double scale, int num_splits,
                           dc_tensor_t *out, dc_tensor_t *lse, void *stream) {
    AttnProblem p;
    int st = fill_problem(q, k, v, 0, has_scale, scale, p);
    if (!st) st = fill_mask(mask, p);
    if (!st) st = check_out(out, lse, p);
    if (st) return st;
    if (p.L != 1) return fail(DC_ERR_VALUE, "decode takes a query length of 1");
    p.out = static_cast<float *>(out->data);
    p.lse = static_cast<float *>(lse->data);
    copy_strides(out, p.os, 4);
    copy_strides(lse, p.ls, 3);
    if (!decode_supported(p))
        return fail(DC_ERR_UNSUPPORTED,
                    "decode needs head dim 64 or 128, E == Ev, unit-stride rows on 16-byte "
                    "boundaries; use dc_sdpa_fwd");
    if (p.B == 0 || p.H == 0) return DC_OK;
    const int splits = num_splits > 0 ? (num_splits > 1024 ? 1024 : num_splits) : decode_pick_splits(p);
    const size_t need = decode_workspace_bytes(p.B, p.H, p.Ev, splits);
    if (need > (size_t)DC_DECODE_NOALLOC_SCRATCH_BYTES)
        return fail(DC_ERR_VALUE,
                    "dc_sdpa_decode_noalloc: " + std::to_string(splits) + " splits over " +
                        std::to_string(p.B * p.H) + " (batch, head) rows need " +
                        std::to_string(need) + " bytes of scratch, more than its fixed " +
                        std::to_string((size_t)DC_DECODE_NOALLOC_SCRATCH_BYTES) +
                        "; pass fewer splits or call dc_sdpa_decode with a workspace");
    if ((st = device_ok())) return st;
    void *scratch = nullptr;
    if ((st = decode_scratch(&scratch))) return st;
    return decode_forward(p, splits, scratch, static_cast<cudaStream_t>(stream));
}

int dc_attn_merge(dc_tensor_t *out_acc, dc_tensor_t *lse_acc, const dc_tensor_t *out_part,
                  const dc_tensor_t *lse_part, void *stream) {
    if (!is_f32(out_acc, 4) || !is_f32(out_part, 4) || !is_f32(lse_acc, 3) || !is_f32(lse_part, 3))
        return fail(DC_ERR_VALUE, "merge takes float32 (B,H,L,Ev) outputs and (B,H,L) logsumexps");
    const int64_t *s = out_acc->sizes;
    if (!sizes_are(out_part, {s[0], s[1], s[2], s[3]}) || !sizes_are(lse_acc, {s[0], s[1], s[2]}) ||
        !sizes_are(lse_part, {s[0], s[1], s[2]}))
        return fail(DC_ERR_VALUE, "merge shapes do not match");
    if (s[0] * s[1] * s[2] == 0) return DC_OK;
    int st = device_ok();
    if (st) return st;
    MergeStrides ms{};
    copy_strides(out_acc, ms.oas, 4);
    copy_strides(lse_acc, ms.las, 3);
    copy_strides(out_part, ms.ops, 4);
    copy_strides(lse_part, ms.lps, 3);
    return merge(static_cast<float *>(out_acc->data), static_cast<float *>(lse_acc->data),
                 static_cast<const float *>(out_part->data),
                 static_cast<const float *>(lse_part->data), s[0], s[1], s[2], s[3], ms,
                 static_cast<cudaStream_t>(stream));
}

static int attn_probs_impl(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *lse,
                           const dc_tensor_t *mask, int causal, int has_scale, double scale,
                           const uint32_t *keep_bits, float keep_scale, bool dropout, int average_heads,
                           dc_tensor_t *probs, void *stream) {
    AttnProblem p;
    int st = fill_problem(q, k, k, causal, has_scale, scale, p);
    if (!st) st = fill_mask(mask, p);
    if (!st && dropout) st = set_keep(p, keep_bits, keep_scale);
    if (st) return st;
    if (!is_f32(lse, 3) || !sizes_are(lse, {p.B, p.H, p.L}))
        return fail(DC_ERR_VALUE, "logsumexp must be float32 (B, H, L)");
    int64_t ps[4];
    if (average_heads) {
        if (!is_f32(probs, 3) || !sizes_are(probs, {p.B, p.L, p.S}))
            return fail(DC_ERR_VALUE, "averaged probabilities must be float32 (B, L, S)");
        ps[0] = probs->strides[0];
        ps[1] = 0;
        ps[2] = probs->strides[1];
        ps[3] = probs->strides[2];
    } else {
        if (!is_f32(probs, 4) || !sizes_are(probs, {p.B, p.H, p.L, p.S}))
            return fail(DC_ERR_VALUE, "probabilities must be float32 (B, H, L, S)");
        for (int i = 0; i < 4; i++) ps[i] = probs->strides[i];
    }
    p.lse = static_cast<float *>(lse->data);
    copy_strides(lse, p.ls, 3);
    if (p.B == 0 || p.L == 0 || p.S == 0) return DC_OK;
    if (p.L > 65535) return fail(DC_ERR_UNSUPPORTED, "probabilities for more than 65535 query rows");
    if ((st = device_ok())) return st;
    return simt_probs(p, static_cast<float *>(probs->data), ps, average_heads,
                      static_cast<cudaStream_t>(stream));
}

int dc_attn_probs(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *lse,
                  const dc_tensor_t *mask, int causal, int has_scale, double scale,
                  int average_heads, dc_tensor_t *probs, void *stream) {
    return attn_probs_impl(q, k, lse, mask, causal, has_scale, scale, nullptr, 0.0f, false, average_heads, probs,
                           stream);
}

int dc_attn_probs_dropout(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *lse,
                          const dc_tensor_t *mask, int causal, int has_scale, double scale,
                          const uint32_t *keep_bits, float keep_scale, int average_heads, dc_tensor_t *probs,
                          void *stream) {
    return attn_probs_impl(q, k, lse, mask, causal, has_scale, scale, keep_bits, keep_scale, true, average_heads,
                           probs, stream);
}

}  // extern "C"
