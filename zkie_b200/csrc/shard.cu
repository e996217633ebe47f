// shard.cu -- one MatMul shard proved on one GPU with the independent stages
// running concurrently (forward C = A W, WHIR base
// commits of W, A and C, and the Op::MatMul GKR proof).
//
// Reference: the committed shard path of zkie-ops (compose.rs:1724-1747 for
// the MatMul arm, compose.rs:2276-2311 for the shard's child transcript,
// pcs/whir.rs:438-469 for each commit).  The reference runs these stages one
// after another on the host; here they are four CUDA streams of one call:
//
//   s1: commit W                        (the largest commit)
//   s2: C = A W, then commit C
//   s3: commit A
//   s0: wait for C, then the GKR proof  (challenges drawn on the host first)
//
// and a single synchronization at the end, when the three roots and the
// proof come back to the host in one transfer each.
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/zkie2.h"
#include "common.cuh"
#include "internal.h"

namespace zk {

namespace {

struct ShardStreams {
    cudaStream_t s[3] = {nullptr, nullptr, nullptr};
    cudaEvent_t fork = nullptr, c_ready = nullptr, join[3] = {nullptr, nullptr, nullptr};
    bool ready = false;
};
std::mutex g_shard_mu;
ShardStreams g_shard[kMaxDevices];

int shard_streams(ShardStreams** out) {
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(g_shard_mu);
    ShardStreams& st = g_shard[d];
    if (!st.ready) {
        for (auto& x : st.s) ZK_TRY(cudaStreamCreateWithFlags(&x, cudaStreamNonBlocking));
        ZK_TRY(cudaEventCreateWithFlags(&st.fork, cudaEventDisableTiming));
        ZK_TRY(cudaEventCreateWithFlags(&st.c_ready, cudaEventDisableTiming));
        for (auto& e : st.join) ZK_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        st.ready = true;
    }
    *out = &st;
    return 0;
}

bool pow2(uint64_t x) { return x && !(x & (x - 1)); }

// Buffers of one WHIR base commit of 2^nv evaluations (LDE 2^(nv-4) x 32).
struct WhirBufs {
    uint64_t *lde, *layers, *scratch;
};

struct ShardLayout {
    WhirBufs w, a, c;
    uint64_t* gkr;
    uint64_t total;
};

ShardLayout shard_layout(uint64_t m, uint64_t k, uint64_t n, uint64_t* base) {
    ShardLayout L{};
    uint64_t off = 0;
    auto take = [&](uint64_t** p, uint64_t cnt) {
        cnt = (cnt + 1) & ~1ull;  // keep 16-byte alignment
        if (base) *p = base + off;
        off += cnt;
    };
    auto whir = [&](WhirBufs* b, uint64_t evals) {
        const uint32_t nv = log2_exact(evals);
        const uint64_t H = 1ull << (nv - 4);
        take(&b->lde, H * 32);
        take(&b->layers, zkie2_merkle_total_digests(H) * 8);
        take(&b->scratch, lde_scratch_elems(nv - 5, 1, 32) + 2);
    };
    whir(&L.w, k * n);
    whir(&L.a, m * k);
    whir(&L.c, m * n);
    take(&L.gkr, op_matmul_scratch_elems(m, k, n));
    L.total = off;
    return L;
}

int whir_enqueue(const uint64_t* d_evals, uint64_t evals, const WhirBufs& b, cudaStream_t s) {
    const uint32_t nv = log2_exact(evals);
    return commit_device(d_evals, nv - 5, 1, 32, b.lde, b.layers, b.scratch, s);
}

}  // namespace
}  // namespace zk

using namespace zk;

extern "C" {

uint64_t zkie2_shard_prove_matmul_scratch_elems(uint64_t m, uint64_t k, uint64_t n) {
    if (!pow2(m) || !pow2(k) || !pow2(n) || m * k < 32 || k * n < 32 || m * n < 32) return 0;
    return shard_layout(m, k, n, nullptr).total;
}

int zkie2_shard_prove_matmul(const uint64_t* d_a, const uint64_t* d_w, uint64_t m, uint64_t k, uint64_t n,
                             const uint64_t* op_ids, uint64_t ops_per_shard, uint64_t shard_index, uint64_t* d_c,
                             uint64_t* h_roots, uint64_t* h_claimed, uint64_t* h_rounds, uint64_t* h_finals,
                             uint64_t* h_claims, uint64_t* d_scratch, cudaStream_t stream) {
    if (!d_a || !d_w || !d_c || !op_ids || !h_roots || !h_claimed || !h_finals || !h_claims || !d_scratch)
        return (int)cudaErrorInvalidValue;
    if (!pow2(m) || !pow2(k) || !pow2(n) || m * k < 32 || k * n < 32 || m * n < 32)
        return (int)cudaErrorInvalidValue;
    const uint32_t lm = log2_exact(m), lk = log2_exact(k), ln = log2_exact(n);
    if (lk && !h_rounds) return (int)cudaErrorInvalidValue;
    ShardStreams* st = nullptr;
    int rc = shard_streams(&st);
    if (rc) return rc;
    rc = p2_ensure_default();
    if (rc) return rc;
    const ShardLayout L = shard_layout(m, k, n, d_scratch);

    // challenges of the shard's child transcript, drawn before any launch
    zkie2_challenger chal;
    zkie2_shard_dag_child(op_ids, 1, ops_per_shard, shard_index, &chal);
    std::vector<uint64_t> u(lm), v(ln), ch(lk);
    for (auto& x : u) x = zkie2_challenger_field(&chal);
    for (auto& x : v) x = zkie2_challenger_field(&chal);
    for (auto& x : ch) x = zkie2_challenger_field(&chal);

    ZK_TRY(cudaEventRecord(st->fork, stream));
    for (auto& s : st->s) ZK_TRY(cudaStreamWaitEvent(s, st->fork, 0));
    // s1: commit W
    rc = whir_enqueue(d_w, k * n, L.w, st->s[0]);
    if (rc) return rc;
    // s2: forward C = A W, then commit C
    rc = matmul_field_dev(d_a, d_w, m, k, n, d_c, st->s[1]);
    if (rc) return rc;
    ZK_TRY(cudaEventRecord(st->c_ready, st->s[1]));
    rc = whir_enqueue(d_c, m * n, L.c, st->s[1]);
    if (rc) return rc;
    // s3: commit A
    rc = whir_enqueue(d_a, m * k, L.a, st->s[2]);
    if (rc) return rc;
    // caller's stream: the GKR proof once C exists
    ZK_TRY(cudaStreamWaitEvent(stream, st->c_ready, 0));
    uint64_t* d_out = nullptr;
    rc = op_matmul_enqueue(d_a, d_w, d_c, m, k, n, u.data(), v.data(), ch.data(), L.gkr, &d_out, stream);
    if (rc) return rc;
    for (int i = 0; i < 3; i++) {
        ZK_TRY(cudaEventRecord(st->join[i], st->s[i]));
        ZK_TRY(cudaStreamWaitEvent(stream, st->join[i], 0));
    }
    // roots: the last digest of each layer buffer (W, A, C)
    const WhirBufs* bufs[3] = {&L.w, &L.a, &L.c};
    const uint64_t evals[3] = {k * n, m * k, m * n};
    for (int i = 0; i < 3; i++) {
        const uint64_t H = evals[i] >> 4;
        const uint64_t* root = bufs[i]->layers + (zkie2_merkle_total_digests(H) - 1) * 8;
        ZK_TRY(cudaMemcpyAsync(h_roots + 8 * i, root, 64, cudaMemcpyDeviceToHost, stream));
    }
    std::vector<uint64_t> out(1 + 3 * lk + 2);
    ZK_TRY(cudaMemcpyAsync(out.data(), d_out, 8 * out.size(), cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaStreamSynchronize(stream));
    *h_claimed = out[0];
    if (lk) std::memcpy(h_rounds, out.data() + 1, 8 * 3 * lk);
    std::memcpy(h_finals, out.data() + 1 + 3 * lk, 16);
    h_claims[0] = h_finals[0];
    h_claims[1] = h_finals[1];
    h_claims[2] = *h_claimed;
    return 0;
}

}  // extern "C"
