// mg.cu -- the multi-GPU context of the C ABI: one split commit and one split
// sumcheck over an NCCL communicator, one process (or one host thread) per
// GPU.  No reference counterpart: the reference commits and proves on one
// device (pcs/merkle_cuda.rs:177-312, common/sumcheck.rs:33-79).
//
// Split commit over G = 2^lg_g ranks (rank g):
//   1. coset g of the LDE rows (rows g, g + G, ...), one H/G-point DFT of the
//      twisted (and, for G > blowup, folded) replicated coefficients;
//   2. its leaf digests;
//   3. one all-to-all of leaf digests (grouped ncclSend / ncclRecv): rank d's
//      contiguous leaf block [d H/G, (d + 1) H/G) holds, from every source s,
//      the rows s + G i of that block, which are a contiguous run of s's
//      digests; an interleave puts them in row order;
//   4. the subtree of the block, an all-gather of the G subtree roots, and
//      the log2 G top levels on every rank: the root of the single-device
//      commit.
// Split sumcheck over G ranks, f and h split by the high variables: the
// first t - log2 G rounds on the local chunks (challenges are known up
// front); the round messages are linear in the pair sums, so ONE all-reduce
// of their 32-bit limbs (exact for up to 2^32 ranks) gives every local
// round's global message; the G folded (f, h) pairs are all-gathered and the
// last log2 G rounds run on every rank.  Same bytes as the single-device
// proof.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2; a process that has
// NCCL loaded already, e.g. through torch, shares that copy), so the
// single-GPU entry points of the library need no NCCL.  NCCL failures return
// kZkMgNcclError + the ncclResult_t.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "../../include/zkie2.h"
#include "common.cuh"
#include "gl64.cuh"
#include "internal.h"

namespace zk {

uint64_t sumcheck_scratch_elems(uint32_t t);
int sumcheck_dev(const uint64_t* d_f, const uint64_t* d_h, uint32_t t, const uint64_t* h_ch, uint64_t* d_rounds,
                 uint64_t* d_finals, uint64_t* d_scratch, cudaStream_t s);
uint64_t lde_coset_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w, uint32_t lg_g);
int lde_coset_launch(const uint64_t* in, uint64_t* out, uint64_t* scratch, uint32_t lg_l, uint32_t lg_blowup,
                     uint64_t w, uint32_t lg_g, uint64_t g, cudaStream_t s);

namespace {

constexpr int kZkMgNcclError = ZKIE2_MG_NCCL_ERROR_BASE;

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*comm_user_rank)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    bool ok = false;
};

std::mutex g_nccl_mu;
NcclApi g_nccl;
bool g_nccl_tried = false;

const NcclApi* nccl() {
    std::lock_guard<std::mutex> g(g_nccl_mu);
    if (!g_nccl_tried) {
        g_nccl_tried = true;
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (h) {
            NcclApi a;
            a.get_unique_id = (decltype(a.get_unique_id))dlsym(h, "ncclGetUniqueId");
            a.comm_init_rank = (decltype(a.comm_init_rank))dlsym(h, "ncclCommInitRank");
            a.comm_destroy = (decltype(a.comm_destroy))dlsym(h, "ncclCommDestroy");
            a.comm_count = (decltype(a.comm_count))dlsym(h, "ncclCommCount");
            a.comm_user_rank = (decltype(a.comm_user_rank))dlsym(h, "ncclCommUserRank");
            a.all_gather = (decltype(a.all_gather))dlsym(h, "ncclAllGather");
            a.all_reduce = (decltype(a.all_reduce))dlsym(h, "ncclAllReduce");
            a.send = (decltype(a.send))dlsym(h, "ncclSend");
            a.recv = (decltype(a.recv))dlsym(h, "ncclRecv");
            a.group_start = (decltype(a.group_start))dlsym(h, "ncclGroupStart");
            a.group_end = (decltype(a.group_end))dlsym(h, "ncclGroupEnd");
            a.ok = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.comm_count && a.comm_user_rank &&
                   a.all_gather && a.all_reduce && a.send && a.recv && a.group_start && a.group_end;
            g_nccl = a;
        }
    }
    return g_nccl.ok ? &g_nccl : nullptr;
}

#define ZK_NCCL(expr)                                              \
    do {                                                           \
        ncclResult_t _r = (expr);                                  \
        if (_r != ncclSuccess) return kZkMgNcclError + (int)_r;    \
    } while (0)

// out[i] = (lo[i] + 2^32 hi[i]) mod p, the ranks' sum of canonical field
// elements reassembled from the all-reduced 32-bit limbs (lo, hi < G 2^32)
__global__ void k_limbs_split(const uint64_t* __restrict__ v, uint64_t n, uint64_t* __restrict__ limbs) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const uint64_t x = v[i];
        limbs[i] = x & 0xFFFFFFFFull;
        limbs[n + i] = x >> 32;
    }
}

__global__ void k_limbs_join(const uint64_t* __restrict__ limbs, uint64_t n, uint64_t* __restrict__ out) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        // lo + hi 2^32 with lo, hi < 2^64: hi 2^32 = (hi_hi 2^64 + hi_lo 2^32), 2^64 = 2^32 - 1 (mod p)
        const uint64_t lo = limbs[i], hi = limbs[n + i];
        const uint64_t hl = hi << 32, hh = hi >> 32;
        uint64_t s = gl_add(gl_canon(lo), gl_canon(hl));
        s = gl_add(s, gl_mul(gl_canon(hh), 0xFFFFFFFFull));
        out[i] = gl_canon(s);
    }
}

// f[r] = pairs[2 r], h[r] = pairs[2 r + 1]
__global__ void k_unpair(const uint64_t* __restrict__ pairs, uint32_t G, uint64_t* __restrict__ f,
                         uint64_t* __restrict__ h) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < G) {
        f[r] = pairs[2 * r];
        h[r] = pairs[2 * r + 1];
    }
}

}  // namespace

}  // namespace zk

using namespace zk;

struct zkie2_mg_ctx {
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = 0, device = -1;
    uint32_t lg_g = 0;
    bool owns = false;
    // streams and events of the host-buffer split commit, made on first use
    cudaStream_t s_in = nullptr, s_nccl = nullptr, s_comp = nullptr, s_out = nullptr;
    cudaEvent_t ev_up[2] = {}, ev_gath[2] = {}, ev_lde[2] = {}, ev_down[2] = {}, ev_a = nullptr, ev_b = nullptr;
    bool pipe_ready = false;
};

namespace {

uint32_t exact_log2(int n) {
    uint32_t r = 0;
    while ((1 << r) < n) r++;
    return (1 << r) == n ? r : 0xFFFFFFFFu;
}

int ctx_check(const zkie2_mg_ctx* c) {
    if (!c || !c->comm) return (int)cudaErrorInvalidValue;
    int d = current_device();
    if (d != c->device) return (int)cudaErrorInvalidDevice;
    return 0;
}

int ctx_finish(ncclComm_t comm, bool owns, zkie2_mg_ctx** out) {
    const NcclApi* api = nccl();
    auto* c = new zkie2_mg_ctx();
    c->comm = comm;
    c->owns = owns;
    c->device = current_device();
    ncclResult_t r = api->comm_count(comm, &c->nranks);
    if (r == ncclSuccess) r = api->comm_user_rank(comm, &c->rank);
    if (r != ncclSuccess) {
        delete c;
        return kZkMgNcclError + (int)r;
    }
    c->lg_g = exact_log2(c->nranks);
    if (c->lg_g == 0xFFFFFFFFu) {  // the split commit needs a power-of-two rank count
        delete c;
        return (int)cudaErrorInvalidValue;
    }
    *out = c;
    return 0;
}

// scratch layout of the split commit: coset NTT scratch, leaf digests, received digests
uint64_t split_commit_coset_elems(uint32_t lg_l, uint32_t lg_b, uint64_t w, uint32_t lg_g) {
    return (lde_coset_scratch_elems(lg_l, lg_b, w, lg_g) + 1) & ~1ull;
}

}  // namespace

extern "C" {

int zkie2_mg_available(void) { return nccl() ? 1 : 0; }

int zkie2_mg_unique_id(uint8_t* h_id) {
    if (!h_id) return (int)cudaErrorInvalidValue;
    const NcclApi* api = nccl();
    if (!api) return (int)cudaErrorSharedObjectInitFailed;
    ncclUniqueId id;
    ZK_NCCL(api->get_unique_id(&id));
    std::memcpy(h_id, id.internal, ZKIE2_MG_UNIQUE_ID_BYTES);
    return 0;
}

int zkie2_mg_init(const uint8_t* h_id, int nranks, int rank, zkie2_mg_ctx** out) {
    if (!h_id || !out || nranks < 1 || rank < 0 || rank >= nranks) return (int)cudaErrorInvalidValue;
    const NcclApi* api = nccl();
    if (!api) return (int)cudaErrorSharedObjectInitFailed;
    ncclUniqueId id;
    std::memcpy(id.internal, h_id, ZKIE2_MG_UNIQUE_ID_BYTES);
    ncclComm_t comm = nullptr;
    ZK_NCCL(api->comm_init_rank(&comm, nranks, id, rank));
    const int rc = ctx_finish(comm, true, out);
    if (rc) api->comm_destroy(comm);
    return rc;
}

int zkie2_mg_init_comm(void* nccl_comm, zkie2_mg_ctx** out) {
    if (!nccl_comm || !out) return (int)cudaErrorInvalidValue;
    if (!nccl()) return (int)cudaErrorSharedObjectInitFailed;
    return ctx_finish(static_cast<ncclComm_t>(nccl_comm), false, out);
}

int zkie2_mg_destroy(zkie2_mg_ctx* ctx) {
    if (!ctx) return 0;
    int rc = 0;
    if (ctx->pipe_ready) {
        for (cudaStream_t st : {ctx->s_in, ctx->s_nccl, ctx->s_comp, ctx->s_out}) cudaStreamDestroy(st);
        for (int i = 0; i < 2; i++)
            for (cudaEvent_t e : {ctx->ev_up[i], ctx->ev_gath[i], ctx->ev_lde[i], ctx->ev_down[i]}) cudaEventDestroy(e);
        cudaEventDestroy(ctx->ev_a);
        cudaEventDestroy(ctx->ev_b);
    }
    if (ctx->owns && ctx->comm) {
        const ncclResult_t r = nccl()->comm_destroy(ctx->comm);
        if (r != ncclSuccess) rc = kZkMgNcclError + (int)r;
    }
    delete ctx;
    return rc;
}

int zkie2_mg_rank(const zkie2_mg_ctx* ctx) { return ctx ? ctx->rank : -1; }
int zkie2_mg_size(const zkie2_mg_ctx* ctx) { return ctx ? ctx->nranks : -1; }

uint64_t zkie2_mg_split_commit_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w, int nranks) {
    const uint32_t lg_g = exact_log2(nranks);
    const uint32_t lg_h = lg_l + lg_blowup;
    if (lg_g == 0xFFFFFFFFu || 2 * lg_g > lg_h || w == 0) return 0;
    const uint64_t n_local = 1ull << (lg_h - lg_g);
    return split_commit_coset_elems(lg_l, lg_blowup, w, lg_g) + 16 * n_local;
}

uint64_t zkie2_mg_top_digests(int nranks) { return nranks < 1 ? 0 : zkie2_merkle_total_digests((uint64_t)nranks); }

int zkie2_mg_split_commit(zkie2_mg_ctx* ctx, const uint64_t* d_coeffs, uint32_t lg_l, uint32_t lg_blowup, uint64_t w,
                          uint64_t* d_lde, uint64_t* d_layers, uint64_t* d_top, uint64_t* d_scratch,
                          uint64_t* h_root, cudaStream_t stream) {
    int rc = ctx_check(ctx);
    if (rc) return rc;
    if (!d_coeffs || !d_lde || !d_layers || !d_top || !d_scratch || !h_root) return (int)cudaErrorInvalidValue;
    const uint32_t lg_h = lg_l + lg_blowup, lg_g = ctx->lg_g;
    if (w == 0 || 2 * lg_g > lg_h || lg_h > 30) return (int)cudaErrorInvalidValue;
    const NcclApi* api = nccl();
    rc = p2_ensure_default();
    if (rc) return rc;
    const int G = ctx->nranks;
    const uint64_t n_local = 1ull << (lg_h - lg_g), per = n_local >> lg_g;
    uint64_t* d_dig = d_scratch + split_commit_coset_elems(lg_l, lg_blowup, w, lg_g);
    uint64_t* d_recv = d_dig + 8 * n_local;
    rc = lde_coset_launch(d_coeffs, d_lde, d_scratch, lg_l, lg_blowup, w, lg_g, (uint64_t)ctx->rank, stream);
    if (!rc) rc = launch_leaf_rows(d_lde, G > 1 ? d_dig : d_layers, 0, n_local, w, stream);
    if (rc) return rc;
    if (G > 1) {
        ZK_NCCL(api->group_start());
        for (int p = 0; p < G; p++) {
            ncclResult_t r = api->send(d_dig + 8 * per * p, 8 * per, ncclUint64, p, ctx->comm, stream);
            if (r == ncclSuccess) r = api->recv(d_recv + 8 * per * p, 8 * per, ncclUint64, p, ctx->comm, stream);
            if (r != ncclSuccess) {
                api->group_end();
                return kZkMgNcclError + (int)r;
            }
        }
        ZK_NCCL(api->group_end());
        rc = zkie2_digests_interleave(d_recv, (uint64_t)G, per, d_layers, stream);
        if (rc) return rc;
    }
    rc = merkle_build_from_leaves(n_local, d_layers, stream);
    if (rc) return rc;
    const uint64_t sub_root = zkie2_merkle_total_digests(n_local) - 1;
    if (G > 1) {
        ZK_NCCL(api->all_gather(d_layers + 8 * sub_root, d_top, 8, ncclUint64, ctx->comm, stream));
        rc = merkle_build_from_leaves((uint64_t)G, d_top, stream);
        if (rc) return rc;
        const uint64_t top_root = zkie2_merkle_total_digests((uint64_t)G) - 1;
        ZK_TRY(cudaMemcpyAsync(h_root, d_top + 8 * top_root, 64, cudaMemcpyDeviceToHost, stream));
    } else {
        ZK_TRY(cudaMemcpyAsync(d_top, d_layers + 8 * sub_root, 64, cudaMemcpyDeviceToDevice, stream));
        ZK_TRY(cudaMemcpyAsync(h_root, d_layers + 8 * sub_root, 64, cudaMemcpyDeviceToHost, stream));
    }
    ZK_TRY(cudaStreamSynchronize(stream));
    return 0;
}

}  // extern "C"

// ---- host buffers in and out, pipelined over column blocks ----------------------------------
// Block j of about four (multiples of 8 columns, the sponge rate): the upload
// of this rank's row slice of the block (copy-in stream), the all-gather of
// the block's rows from every rank (NCCL stream), the block's coset LDE and
// its absorption into every local row's sponge (compute stream; sponge
// states carried in HBM between blocks), and the download of the block's LDE
// rows (copy-out stream) overlap across blocks, two buffer slots deep.  Then
// the digest all-to-all, the subtree, the root all-gather and the top tree,
// and the layers go back to the host.
namespace {

uint64_t mg_col_block(uint64_t w) { return w >= 64 ? ((w + 3) / 4 + 7) / 8 * 8 : w; }

struct MgHostLayout {
    uint64_t part, full, lde, coset, slot, states, dig, recv, layers, top, total;
};

MgHostLayout mg_host_layout(uint32_t lg_l, uint32_t lg_b, uint64_t w, uint32_t lg_g, int G) {
    MgHostLayout L{};
    const uint64_t cw = mg_col_block(w), rows = (1ull << lg_l) >> lg_g;
    const uint64_t n_local = 1ull << (lg_l + lg_b - lg_g);
    auto even = [](uint64_t x) { return (x + 1) & ~1ull; };
    L.part = 0;
    L.full = even(rows * cw);
    L.lde = L.full + even((1ull << lg_l) * cw);
    L.coset = L.lde + even(n_local * cw);
    L.slot = L.coset + split_commit_coset_elems(lg_l, lg_b, cw, lg_g);
    L.states = 2 * L.slot;
    L.dig = L.states + (cw < w ? 16 * n_local : 0);
    L.recv = L.dig + 8 * n_local;
    L.layers = L.recv + 8 * n_local;
    L.top = L.layers + 8 * zkie2_merkle_total_digests(n_local);
    L.total = L.top + 8 * zkie2_merkle_total_digests((uint64_t)G);
    return L;
}

int mg_pipe_ready(zkie2_mg_ctx* c) {
    if (c->pipe_ready) return 0;
    for (cudaStream_t* st : {&c->s_in, &c->s_nccl, &c->s_comp, &c->s_out})
        ZK_TRY(cudaStreamCreateWithFlags(st, cudaStreamNonBlocking));
    for (int i = 0; i < 2; i++)
        for (cudaEvent_t* e : {&c->ev_up[i], &c->ev_gath[i], &c->ev_lde[i], &c->ev_down[i]})
            ZK_TRY(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    ZK_TRY(cudaEventCreateWithFlags(&c->ev_a, cudaEventDisableTiming));
    ZK_TRY(cudaEventCreateWithFlags(&c->ev_b, cudaEventDisableTiming));
    c->pipe_ready = true;
    return 0;
}

// b waits for everything enqueued on a so far
int mg_after(zkie2_mg_ctx* c, cudaStream_t a, cudaStream_t b) {
    ZK_TRY(cudaEventRecord(c->ev_a, a));
    ZK_TRY(cudaStreamWaitEvent(b, c->ev_a, 0));
    return 0;
}

int mg_host_body(zkie2_mg_ctx* c, const uint64_t* h_part, uint32_t lg_l, uint32_t lg_b, uint64_t w,
                 uint64_t* h_lde, uint64_t* h_layers, uint64_t* h_root, uint64_t* S) {
    const NcclApi* api = nccl();
    const int G = c->nranks;
    const uint32_t lg_g = c->lg_g;
    const MgHostLayout L = mg_host_layout(lg_l, lg_b, w, lg_g, G);
    const uint64_t cw = mg_col_block(w), nblk = (w + cw - 1) / cw;
    const uint64_t rows = (1ull << lg_l) >> lg_g, n_local = 1ull << (lg_l + lg_b - lg_g);
    uint64_t* states = S + L.states;
    uint64_t* dig = S + L.dig;
    for (uint64_t j = 0; j < nblk; j++) {
        const int s = (int)(j & 1);
        uint64_t* slot = S + s * L.slot;
        uint64_t *part = slot + L.part, *full = slot + L.full, *lde = slot + L.lde, *scr = slot + L.coset;
        const uint64_t c0 = j * cw, cn = (w - c0) < cw ? (w - c0) : cw;
        // upload this rank's rows of the block (part is free once block j-2 was gathered)
        if (j >= 2) ZK_TRY(cudaStreamWaitEvent(c->s_in, c->ev_gath[s], 0));
        ZK_TRY(cudaMemcpy2DAsync(part, 8 * cn, h_part + c0, 8 * w, 8 * cn, rows, cudaMemcpyHostToDevice, c->s_in));
        ZK_TRY(cudaEventRecord(c->ev_up[s], c->s_in));
        // every rank's rows of the block (full is free once block j-2's LDE read it)
        ZK_TRY(cudaStreamWaitEvent(c->s_nccl, c->ev_up[s], 0));
        if (j >= 2) ZK_TRY(cudaStreamWaitEvent(c->s_nccl, c->ev_lde[s], 0));
        if (G > 1) {
            ZK_NCCL(api->all_gather(part, full, rows * cn, ncclUint64, c->comm, c->s_nccl));
        } else {
            ZK_TRY(cudaMemcpyAsync(full, part, 8 * rows * cn, cudaMemcpyDeviceToDevice, c->s_nccl));
        }
        ZK_TRY(cudaEventRecord(c->ev_gath[s], c->s_nccl));
        // the block's coset LDE (lde is free once block j-2's rows were downloaded), then its absorption
        ZK_TRY(cudaStreamWaitEvent(c->s_comp, c->ev_gath[s], 0));
        if (j >= 2 && h_lde) ZK_TRY(cudaStreamWaitEvent(c->s_comp, c->ev_down[s], 0));
        int rc = lde_coset_launch(full, lde, scr, lg_l, lg_b, cn, lg_g, (uint64_t)c->rank, c->s_comp);
        if (rc) return rc;
        ZK_TRY(cudaEventRecord(c->ev_lde[s], c->s_comp));
        rc = nblk > 1 ? launch_leaf_absorb(lde, cn, 0, cn, n_local, states, dig, j == 0, j + 1 == nblk, c->s_comp)
                      : launch_leaf_rows(lde, dig, 0, n_local, cn, c->s_comp);
        if (rc) return rc;
        if (h_lde) {
            ZK_TRY(cudaStreamWaitEvent(c->s_out, c->ev_lde[s], 0));
            ZK_TRY(cudaMemcpy2DAsync(h_lde + c0, 8 * w, lde, 8 * cn, 8 * cn, n_local, cudaMemcpyDeviceToHost,
                                     c->s_out));
            ZK_TRY(cudaEventRecord(c->ev_down[s], c->s_out));
        }
    }
    // the digest exchange, the subtree and the top levels
    uint64_t* layers = S + L.layers;
    uint64_t* top = S + L.top;
    const uint64_t per = n_local >> lg_g;
    int rc = 0;
    if (G > 1) {
        uint64_t* recv = S + L.recv;
        rc = mg_after(c, c->s_comp, c->s_nccl);
        if (rc) return rc;
        ZK_NCCL(api->group_start());
        for (int p = 0; p < G; p++) {
            ncclResult_t r = api->send(dig + 8 * per * p, 8 * per, ncclUint64, p, c->comm, c->s_nccl);
            if (r == ncclSuccess) r = api->recv(recv + 8 * per * p, 8 * per, ncclUint64, p, c->comm, c->s_nccl);
            if (r != ncclSuccess) {
                api->group_end();
                return kZkMgNcclError + (int)r;
            }
        }
        ZK_NCCL(api->group_end());
        rc = mg_after(c, c->s_nccl, c->s_comp);
        if (!rc) rc = zkie2_digests_interleave(recv, (uint64_t)G, per, layers, c->s_comp);
    } else {
        rc = (int)cudaMemcpyAsync(layers, dig, 64 * n_local, cudaMemcpyDeviceToDevice, c->s_comp);
    }
    if (!rc) rc = merkle_build_from_leaves(n_local, layers, c->s_comp);
    if (rc) return rc;
    const uint64_t sub_root = zkie2_merkle_total_digests(n_local) - 1;
    if (G > 1) {
        rc = mg_after(c, c->s_comp, c->s_nccl);
        if (rc) return rc;
        ZK_NCCL(api->all_gather(layers + 8 * sub_root, top, 8, ncclUint64, c->comm, c->s_nccl));
        rc = mg_after(c, c->s_nccl, c->s_comp);
        if (!rc) rc = merkle_build_from_leaves((uint64_t)G, top, c->s_comp);
        if (rc) return rc;
        const uint64_t top_root = zkie2_merkle_total_digests((uint64_t)G) - 1;
        ZK_TRY(cudaMemcpyAsync(h_root, top + 8 * top_root, 64, cudaMemcpyDeviceToHost, c->s_comp));
    } else {
        ZK_TRY(cudaMemcpyAsync(h_root, layers + 8 * sub_root, 64, cudaMemcpyDeviceToHost, c->s_comp));
    }
    if (h_layers)
        ZK_TRY(cudaMemcpyAsync(h_layers, layers, 64 * (sub_root + 1), cudaMemcpyDeviceToHost, c->s_comp));
    return 0;
}

}  // namespace

extern "C" {

uint64_t zkie2_mg_split_commit_host_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w, int nranks) {
    const uint32_t lg_g = exact_log2(nranks);
    if (lg_g == 0xFFFFFFFFu || 2 * lg_g > lg_l + lg_blowup || lg_g > lg_l || w == 0) return 0;
    return mg_host_layout(lg_l, lg_blowup, w, lg_g, nranks).total;
}

int zkie2_mg_split_commit_host(zkie2_mg_ctx* ctx, const uint64_t* h_part, uint32_t lg_l, uint32_t lg_blowup,
                               uint64_t w, uint64_t* h_lde, uint64_t* h_layers, uint64_t* h_root,
                               uint64_t* d_scratch) {
    int rc = ctx_check(ctx);
    if (rc) return rc;
    const uint32_t lg_h = lg_l + lg_blowup;
    if (!h_part || !h_root || !d_scratch || w == 0 || 2 * ctx->lg_g > lg_h || ctx->lg_g > lg_l || lg_h > 30)
        return (int)cudaErrorInvalidValue;
    rc = p2_ensure_default();
    if (!rc) rc = mg_pipe_ready(ctx);
    if (rc) return rc;
    // the caller's earlier work on the legacy stream (e.g. filling the scratch) comes first
    if (cudaEventRecord(ctx->ev_b, 0) == cudaSuccess)
        for (cudaStream_t st : {ctx->s_in, ctx->s_nccl, ctx->s_comp, ctx->s_out}) cudaStreamWaitEvent(st, ctx->ev_b, 0);
    rc = mg_host_body(ctx, h_part, lg_l, lg_blowup, w, h_lde, h_layers, h_root, d_scratch);
    // every stream drains before returning, also after an error part-way
    for (cudaStream_t st : {ctx->s_in, ctx->s_nccl, ctx->s_comp, ctx->s_out}) {
        const cudaError_t e = cudaStreamSynchronize(st);
        if (!rc && e != cudaSuccess) rc = (int)e;
    }
    return rc;
}

uint64_t zkie2_mg_split_sumcheck_scratch_elems(uint32_t t, int nranks) {
    const uint32_t lg_g = exact_log2(nranks);
    if (lg_g == 0xFFFFFFFFu || lg_g > t) return 0;
    const uint32_t t_loc = t - lg_g;
    const uint64_t a = sumcheck_scratch_elems(t_loc), b = sumcheck_scratch_elems(lg_g);
    // local rounds + finals, limbs, gathered pairs, f and h of the top rounds, top-round scratch
    return 3ull * t + 2 + 6ull * t + 2ull * nranks + 2ull * nranks + 2 + (a > b ? a : b) + 8;
}

int zkie2_mg_split_sumcheck(zkie2_mg_ctx* ctx, const uint64_t* d_f, const uint64_t* d_h, uint32_t t,
                            const uint64_t* h_ch, uint64_t* h_rounds, uint64_t* h_finals, uint64_t* d_scratch,
                            cudaStream_t stream) {
    int rc = ctx_check(ctx);
    if (rc) return rc;
    const uint32_t lg_g = ctx->lg_g;
    if (!d_f || !d_h || !h_finals || !d_scratch || lg_g > t || (t && (!h_ch || !h_rounds)))
        return (int)cudaErrorInvalidValue;
    const NcclApi* api = nccl();
    const int G = ctx->nranks;
    const uint32_t t_loc = t - lg_g;
    uint64_t* d_rounds = d_scratch;                 // 3 t
    uint64_t* d_fin_loc = d_rounds + 3ull * t;      // 2
    uint64_t* d_limbs = d_fin_loc + 2;              // 2 * 3 t_loc
    uint64_t* d_pairs = d_limbs + 6ull * t;         // 2 G
    uint64_t* d_fg = d_pairs + 2ull * G;            // G
    uint64_t* d_hg = d_fg + G;                      // G
    uint64_t* d_fin = d_hg + G;                     // 2
    uint64_t* d_scr = d_fin + 2;
    d_scr += (reinterpret_cast<uintptr_t>(d_scr) / 8) & 1;  // 16-byte alignment for the sumcheck's vector loads
    rc = sumcheck_dev(d_f, d_h, t_loc, h_ch, d_rounds, d_fin_loc, d_scr, stream);
    if (rc) return rc;
    if (G > 1) {
        const uint64_t n = 3ull * t_loc;
        if (n) {
            k_limbs_split<<<(unsigned)ceil_div(n, 256), 256, 0, stream>>>(d_rounds, n, d_limbs);
            ZK_LAUNCH_CHECK();
            ZK_NCCL(api->all_reduce(d_limbs, d_limbs, 2 * n, ncclUint64, ncclSum, ctx->comm, stream));
            k_limbs_join<<<(unsigned)ceil_div(n, 256), 256, 0, stream>>>(d_limbs, n, d_rounds);
            ZK_LAUNCH_CHECK();
        }
        ZK_NCCL(api->all_gather(d_fin_loc, d_pairs, 2, ncclUint64, ctx->comm, stream));
        k_unpair<<<(unsigned)ceil_div((uint64_t)G, 256), 256, 0, stream>>>(d_pairs, (uint32_t)G, d_fg, d_hg);
        ZK_LAUNCH_CHECK();
        rc = sumcheck_dev(d_fg, d_hg, lg_g, h_ch + t_loc, d_rounds + 3ull * t_loc, d_fin, d_scr, stream);
        if (rc) return rc;
    } else {
        d_fin = d_fin_loc;
    }
    if (t) ZK_TRY(cudaMemcpyAsync(h_rounds, d_rounds, 24ull * t, cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaMemcpyAsync(h_finals, d_fin, 16, cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaStreamSynchronize(stream));
    return 0;
}

}  // extern "C"
