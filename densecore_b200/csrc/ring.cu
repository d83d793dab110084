// ring.cu -- dc_ring_sdpa_fwd: sequence-parallel ring attention (forward) over the ranks of a
// caller's NCCL communicator.
//
// DenseCore's flash forward (src/torch_attention.rs:146-284) runs every (batch, head) task over
// the whole key range on one host. For the long-context causal prefill this entry point splits
// the sequence over the P ranks of a communicator and passes K/V blocks around a ring; each
// rank's result equals that forward on the full sequence, restricted to its own query rows.
//
// Layout (zig-zag, for causal balance): the sequence is cut into 2P chunks of C rows; rank r
// holds query, key and value chunks r and 2P-1-r back to back as its local (B, H, 2C, E) shard.
// Step 0 is a causal attention of the local rows over the local keys. At step t > 0 the rank
// holds the keys and values rank s = (r - t) mod P started with; under causal masking the step
// reduces to one non-causal call: all 2C local rows against the first C keys when s < r, or the
// last C local rows against all 2C keys when s > r (without causal masking: all rows against
// all keys). Each partial result is folded into (out, lse) by the logsumexp merge.
//
// K and V travel packed in one (2, B, Hkv, 2C, E) buffer of the caller's workspace: at step t
// the rank sends the block it holds to rank r+1 and receives the next one from rank r-1 into
// the second buffer, with ncclSend / ncclRecv in one group on a side stream of the library's.
// The transfer that feeds step t + 1 runs beside step t's attention on the caller's stream;
// the side stream has the device's greatest priority, so NCCL's blocks are scheduled ahead
// of the attention blocks still waiting for an SM.
// No kernel reads another GPU's memory: the only traffic between GPUs is NCCL's.
//
// libnccl is not a link-time dependency of the library: its entry points are resolved at the
// first ring call from the libnccl.so.2 already loaded in the process (the one the caller made
// its communicator with), or loaded by that name.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace dc {
namespace {

struct NcclApi {
    decltype(&ncclSend) send = nullptr;
    decltype(&ncclRecv) recv = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclCommCount) count = nullptr;
    decltype(&ncclCommUserRank) user_rank = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    bool ok = false;
    std::string why;
};

const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char *e = dlerror();
            api.why = std::string("cannot load libnccl.so.2: ") + (e ? e : "unknown error");
            return;
        }
        api.send = reinterpret_cast<decltype(api.send)>(dlsym(h, "ncclSend"));
        api.recv = reinterpret_cast<decltype(api.recv)>(dlsym(h, "ncclRecv"));
        api.group_start = reinterpret_cast<decltype(api.group_start)>(dlsym(h, "ncclGroupStart"));
        api.group_end = reinterpret_cast<decltype(api.group_end)>(dlsym(h, "ncclGroupEnd"));
        api.count = reinterpret_cast<decltype(api.count)>(dlsym(h, "ncclCommCount"));
        api.user_rank = reinterpret_cast<decltype(api.user_rank)>(dlsym(h, "ncclCommUserRank"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.send && api.recv && api.group_start && api.group_end && api.count && api.user_rank &&
                 api.error_string;
        if (!api.ok) api.why = "libnccl.so.2 lacks ncclSend / ncclRecv / ncclGroupStart / ncclGroupEnd";
    });
    return api;
}

int nccl_fail(const NcclApi &api, ncclResult_t r, const char *what) {
    return fail(DC_ERR_RUNTIME, std::string("ring attention: ") + what + ": " + api.error_string(r));
}

constexpr int kSideRoleRing = 1;

// Sub-view of rows [r0, r0 + n) along dim 2 of a 4-D view (or of a 3-D lse view).
dc_tensor_t rows(const dc_tensor_t &t, int64_t r0, int64_t n) {
    dc_tensor_t v = t;
    v.data = static_cast<char *>(t.data) + r0 * t.strides[2] * (int64_t)sizeof(float);
    v.sizes[2] = n;
    return v;
}

dc_tensor_t contiguous_view(float *data, int64_t a, int64_t b, int64_t c, int64_t d, int ndim) {
    dc_tensor_t v{};
    v.data = data;
    v.dtype = DC_F32;
    v.ndim = ndim;
    const int64_t s[4] = {a, b, c, d};
    int64_t st = 1;
    for (int i = ndim - 1; i >= 0; i--) {
        v.sizes[i] = s[i];
        v.strides[i] = st;
        st *= s[i];
    }
    return v;
}

bool is_contiguous4(const dc_tensor_t *t) {
    return t->ndim == 4 && t->strides[3] == 1 && t->strides[2] == t->sizes[3] &&
           t->strides[1] == t->sizes[2] * t->sizes[3] && t->strides[0] == t->sizes[1] * t->sizes[2] * t->sizes[3];
}

}  // namespace
}  // namespace dc

using namespace dc;

extern "C" {

size_t dc_ring_sdpa_fwd_workspace_size(int64_t batch, int64_t heads, int64_t kv_heads, int64_t local_len,
                                       int64_t head_dim) {
    if (batch <= 0 || heads <= 0 || kv_heads <= 0 || local_len <= 0 || head_dim <= 0) return 0;
    const size_t kv = 2 * (size_t)batch * kv_heads * local_len * head_dim;   // one packed K/V block
    const size_t part = (size_t)batch * heads * local_len * (head_dim + 1);  // partial out + lse
    return ((2 * kv + part) * sizeof(float) + 255) / 256 * 256;
}

int dc_ring_sdpa_fwd(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *v, int causal,
                     int has_scale, double scale, int precision, struct ncclComm *comm, dc_tensor_t *out,
                     dc_tensor_t *lse, void *workspace, size_t workspace_bytes, void *stream) {
    if (!q || !k || !v || !out || !lse)
        return fail(DC_ERR_VALUE, "ring attention: q, k, v, out and lse are required");
    if (q->ndim != 4 || k->ndim != 4 || v->ndim != 4 || q->dtype != DC_F32 || k->dtype != DC_F32 ||
        v->dtype != DC_F32)
        return fail(DC_ERR_VALUE, "ring attention takes (B, H, L, E) float32 shards");
    for (int i = 0; i < 4; i++)
        if (k->sizes[i] != v->sizes[i])
            return fail(DC_ERR_VALUE, "ring attention needs k and v of the same shape");
    const int64_t B = q->sizes[0], H = q->sizes[1], L2 = q->sizes[2], E = q->sizes[3], Hkv = k->sizes[1];
    if (k->sizes[0] != B || k->sizes[2] != L2 || k->sizes[3] != E || Hkv <= 0 || H % Hkv)
        return fail(DC_ERR_VALUE, "ring attention needs local query and key shards of the same length, batch and "
                                  "head dim (and H % Hkv == 0)");
    if (L2 % 2) return fail(DC_ERR_VALUE, "ring attention needs an even local length (two zig-zag chunks)");
    if (!is_contiguous4(k) || !is_contiguous4(v))
        return fail(DC_ERR_VALUE, "ring attention sends k and v as they are: they must be contiguous");
    if (!comm) return fail(DC_ERR_VALUE, "ring attention: the NCCL communicator is null");
    const size_t need = dc_ring_sdpa_fwd_workspace_size(B, H, Hkv, L2, E);
    if (need && (!workspace || workspace_bytes < need))
        return fail(DC_ERR_VALUE, "ring attention: workspace of " + std::to_string(workspace_bytes) + " bytes, " +
                                      std::to_string(need) + " needed");
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return fail(DC_ERR_VALUE, "ring attention: the workspace must be 256-byte aligned");
    const NcclApi &api = nccl();
    if (!api.ok) return fail(DC_ERR_RUNTIME, "ring attention: " + api.why);
    int world = 0, rank = 0;
    ncclResult_t nr = api.count(comm, &world);
    if (nr == ncclSuccess) nr = api.user_rank(comm, &rank);
    if (nr != ncclSuccess) return nccl_fail(api, nr, "communicator size / rank");
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    // One rank: the whole sequence is local.
    if (world == 1 || B * H * L2 == 0)
        return dc_sdpa_fwd(q, k, v, nullptr, causal, has_scale, scale, precision, out, lse, stream);
    int st = DC_OK;

    const int64_t C = L2 / 2;
    const size_t kv_elems = 2 * (size_t)B * Hkv * L2 * E;
    float *bufs[2] = {static_cast<float *>(workspace), static_cast<float *>(workspace) + kv_elems};
    float *part_o = bufs[1] + kv_elems;
    float *part_l = part_o + (size_t)B * H * L2 * E;
    const int next = (rank + 1) % world, prev = (rank + world - 1) % world;
    cudaStream_t side = nullptr;
    if ((st = side_stream(s, kSideRoleRing, &side))) return st;
    StreamJoin join(s, side);  // the side stream joins the caller's on every return

    // Transfer j (1 <= j < P) brings the block of rank (rank - j) into bufs[j % 2]: this rank
    // sends the block it holds (k and v themselves for j = 1) and receives the next. It is
    // enqueued before the attention of step j - 1, so the two overlap; it starts once step
    // j - 2's attention, the last reader of bufs[j % 2], is done, and step j waits for it.
    auto transfer = [&](int j) -> int {
        int rc = stream_edge(s, side);  // the buffer's last reader is done
        if (rc) return rc;
        float *recv_buf = bufs[j % 2];
        const size_t half = kv_elems / 2;
        ncclResult_t r = api.group_start();
        if (r == ncclSuccess) {
            if (j == 1) {
                r = api.send(k->data, half, ncclFloat32, next, comm, side);
                if (r == ncclSuccess) r = api.send(v->data, half, ncclFloat32, next, comm, side);
                if (r == ncclSuccess) r = api.recv(recv_buf, half, ncclFloat32, prev, comm, side);
                if (r == ncclSuccess) r = api.recv(recv_buf + half, half, ncclFloat32, prev, comm, side);
            } else {
                r = api.send(bufs[(j - 1) % 2], kv_elems, ncclFloat32, next, comm, side);
                if (r == ncclSuccess) r = api.recv(recv_buf, kv_elems, ncclFloat32, prev, comm, side);
            }
            const ncclResult_t ge = api.group_end();
            if (r == ncclSuccess) r = ge;
        }
        return r == ncclSuccess ? DC_OK : nccl_fail(api, r, "send / recv of the K/V block");
    };

    // Step 0: causal (or full) attention of the local rows over the local keys, beside transfer 1.
    if ((st = transfer(1))) return st;
    if ((st = dc_sdpa_fwd(q, k, v, nullptr, causal, has_scale, scale, precision, out, lse, stream))) return st;

    for (int t = 1; t < world; t++) {
        // The side stream's tail is transfer t here: this step's attention reads its block.
        if ((st = stream_edge(side, s))) return st;
        if (t + 1 < world && (st = transfer(t + 1))) return st;

        const int src = (rank - t + world) % world;
        float *blk = bufs[t % 2];
        dc_tensor_t kk = contiguous_view(blk, B, Hkv, L2, E, 4);
        dc_tensor_t vv = contiguous_view(blk + kv_elems / 2, B, Hkv, L2, E, 4);
        if (!causal || src < rank) {
            // All local rows against the first C keys of the block (all of them without causal).
            const int64_t nk = causal ? C : L2;
            dc_tensor_t ks = rows(kk, 0, nk), vs = rows(vv, 0, nk);
            dc_tensor_t po = contiguous_view(part_o, B, H, L2, E, 4), pl = contiguous_view(part_l, B, H, L2, 0, 3);
            if ((st = dc_sdpa_fwd(q, &ks, &vs, nullptr, 0, has_scale, scale, precision, &po, &pl, stream))) return st;
            if ((st = dc_attn_merge(out, lse, &po, &pl, stream))) return st;
        } else {
            // The last C local rows against every key of the block.
            dc_tensor_t qs = rows(*q, C, C), os = rows(*out, C, C), ls = rows(*lse, C, C);
            dc_tensor_t po = contiguous_view(part_o, B, H, C, E, 4), pl = contiguous_view(part_l, B, H, C, 0, 3);
            if ((st = dc_sdpa_fwd(&qs, &kk, &vv, nullptr, 0, has_scale, scale, precision, &po, &pl, stream)))
                return st;
            if ((st = dc_attn_merge(&os, &ls, &po, &pl, stream))) return st;
        }
    }
    return join.join();
}

}  // extern "C"
