// commit.cu -- the shard commit stage: zero-padded LDE + Poseidon2 Merkle tree
// over the rows, in one device pipeline.
//
// The reference runs this as two host round trips (pcs/dft_cuda.rs:184-221
// uploads the coefficients, downloads the LDE; pcs/merkle_cuda.rs:177-312
// uploads the LDE again and downloads the digest layers).  Here the LDE stays
// in HBM between the transform and the hashing; only the final results cross
// PCIe, and the download of the LDE overlaps the hashing.
#include <mutex>

#include "../../include/zkie2.h"
#include "common.cuh"
#include "internal.h"

namespace zk {

namespace {

constexpr int kMaxChunks = 8;  // column blocks of the pipelined host commit

// Per-device state of zkie2_commit_host.  The streams and events are shared by
// every call on the device, so `call` serialises whole calls: a second host
// thread waits instead of re-recording an event between another call's record
// and its wait.  `pool` is the library's own stream-ordered pool: it caches
// freed blocks across calls without changing the device's default pool, which
// the caller's allocator (torch, cudaMallocAsync users) may rely on.
struct DevStreams {
    cudaStream_t compute = nullptr, copy = nullptr, copy_out = nullptr, hash = nullptr;
    cudaEvent_t lde_ready = nullptr;
    cudaEvent_t in_ready[kMaxChunks] = {}, chunk_lde[kMaxChunks] = {};
    cudaMemPool_t pool = nullptr;
    std::mutex call;
    bool ready = false;
};
std::mutex g_streams_mu;
DevStreams g_streams[kMaxDevices];

int get_streams(DevStreams** out) {
    int d = current_device();
    if (d < 0 || d >= kMaxDevices) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(g_streams_mu);
    DevStreams& s = g_streams[d];
    if (!s.ready) {
        ZK_TRY(cudaStreamCreateWithFlags(&s.compute, cudaStreamNonBlocking));
        ZK_TRY(cudaStreamCreateWithFlags(&s.copy, cudaStreamNonBlocking));
        ZK_TRY(cudaStreamCreateWithFlags(&s.copy_out, cudaStreamNonBlocking));
        ZK_TRY(cudaStreamCreateWithFlags(&s.hash, cudaStreamNonBlocking));
        ZK_TRY(cudaEventCreateWithFlags(&s.lde_ready, cudaEventDisableTiming));
        for (int i = 0; i < kMaxChunks; i++) {
            ZK_TRY(cudaEventCreateWithFlags(&s.in_ready[i], cudaEventDisableTiming));
            ZK_TRY(cudaEventCreateWithFlags(&s.chunk_lde[i], cudaEventDisableTiming));
        }
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = d;
        ZK_TRY(cudaMemPoolCreate(&s.pool, &props));
        uint64_t thr = ~0ull;  // keep freed blocks cached across calls (this pool only)
        ZK_TRY(cudaMemPoolSetAttribute(s.pool, cudaMemPoolAttrReleaseThreshold, &thr));
        s.ready = true;
    }
    *out = &s;
    return 0;
}

}  // namespace

// LDE (rows >= rows_valid of the L-row input are zero) followed by the tree.
int commit_device(const uint64_t* d_in, uint32_t lg_l, uint32_t lg_blowup, uint64_t w,
                  uint64_t* d_lde, uint64_t* d_layers, uint64_t* d_scratch, cudaStream_t s) {
    int rc = p2_ensure_default();
    if (rc) return rc;
    rc = lde_launch(d_in, d_lde, d_scratch, lg_l, lg_blowup, w, s);
    if (rc) return rc;
    const uint64_t H = 1ull << (lg_l + lg_blowup);
    return merkle_build(d_lde, H, w, d_layers, s);
}

}  // namespace zk

using namespace zk;

extern "C" {

uint64_t zkie2_commit_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w) {
    return lde_scratch_elems(lg_l, lg_blowup, w);
}

int zkie2_commit(const uint64_t* d_coeffs, uint32_t lg_l, uint32_t lg_blowup, uint64_t w,
                 uint64_t* d_lde, uint64_t* d_layers, uint64_t* d_scratch, cudaStream_t stream) {
    if (w == 0) return (int)cudaErrorInvalidValue;
    return commit_device(d_coeffs, lg_l, lg_blowup, w, d_lde, d_layers, d_scratch, stream);
}

// WHIR base commit (pcs/whir.rs:438-469): 2^n evaluations as a row-major
// 2^(n-5) x 32 matrix (width 2^folding, folding factor 5), zero-padded to
// twice the height (starting_log_inv_rate 1), DFT per column, Merkle over rows.
int zkie2_whir_commit(const uint64_t* d_evals, uint32_t n, uint64_t* d_lde, uint64_t* d_layers,
                      uint64_t* d_scratch, cudaStream_t stream) {
    if (n < 5) return (int)cudaErrorInvalidValue;
    return commit_device(d_evals, n - 5, 1, 32, d_lde, d_layers, d_scratch, stream);
}

uint64_t zkie2_whir_scratch_elems(uint32_t n) { return n < 5 ? 0 : lde_scratch_elems(n - 5, 1, 32); }

// commit_extension (vendor/p3-whir/src/pcs/committer/writer.rs:21-86, Suffix
// order): the 2^n extension-field evaluations (degree-2 binomial extension,
// each element stored as its two base coefficients c0, c1) fill the first
// 2^(n-5) rows of a (2^(n-5) << log_inv_rate) x 32 EF matrix, zero rows
// below, and every EF column is DFT'd.  The twiddles are base-field elements,
// so the EF DFT acts on each coefficient column separately
// (dft_algebra_batch); and ExtensionMmcs hashes each row as its 64 base
// coefficients.  Together: an LDE of the 2^(n-5) x 64 base matrix at
// blowup 2^log_inv_rate and the Merkle tree over its 64-wide rows.
int zkie2_commit_extension(const uint64_t* d_evals, uint32_t n, uint32_t log_inv_rate, uint64_t* d_lde,
                           uint64_t* d_layers, uint64_t* d_scratch, cudaStream_t stream) {
    if (n < 5) return (int)cudaErrorInvalidValue;
    return commit_device(d_evals, n - 5, log_inv_rate, 64, d_lde, d_layers, d_scratch, stream);
}

uint64_t zkie2_commit_extension_scratch_elems(uint32_t n, uint32_t log_inv_rate) {
    return n < 5 ? 0 : lde_scratch_elems(n - 5, log_inv_rate, 64);
}

// Commit of a matrix whose LDE does not fit in HBM next to its inputs (the
// 256 x 2^24 cases of the raw-commit sweep need 64-128 GiB of LDE plus the
// same again of NTT scratch): the LDE rows are produced one coset at a time.
// Coset c of C = 2^lg_c holds the rows i = c + C*i' (zkie2_lde_coset, the
// per-rank step of the multi-GPU split commit); its leaf digests go to a
// staging area in coset-major order, the coset's LDE buffer is reused for the
// next coset, and one interleave puts the H digests in row order before the
// tree.  Same root and layers as zkie2_commit; the LDE is not kept.
uint64_t zkie2_commit_cosets_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w, uint32_t lg_c) {
    const uint32_t lg_h = lg_l + lg_blowup;
    if (2 * lg_c > lg_h) return 0;
    const uint64_t H = 1ull << lg_h;
    return (H >> lg_c) * w + zkie2_lde_coset_scratch_elems(lg_l, lg_blowup, w, lg_c) + 8 * H;
}

int zkie2_commit_cosets(const uint64_t* d_coeffs, uint32_t lg_l, uint32_t lg_blowup, uint64_t w, uint32_t lg_c,
                        uint64_t* d_layers, uint64_t* d_scratch, cudaStream_t stream) {
    const uint32_t lg_h = lg_l + lg_blowup;
    if (!d_coeffs || !d_layers || !d_scratch || w == 0 || 2 * lg_c > lg_h) return (int)cudaErrorInvalidValue;
    int rc = p2_ensure_default();
    if (rc) return rc;
    const uint64_t H = 1ull << lg_h, rows = H >> lg_c, C = 1ull << lg_c;
    uint64_t* d_lde = d_scratch;
    uint64_t* d_ntt = d_lde + rows * w;
    uint64_t* d_stage = d_ntt + zkie2_lde_coset_scratch_elems(lg_l, lg_blowup, w, lg_c);
    for (uint64_t c = 0; c < C; c++) {
        rc = zkie2_lde_coset(d_coeffs, d_lde, d_ntt, lg_l, lg_blowup, w, lg_c, c, stream);
        if (!rc) rc = launch_leaf_rows(d_lde, d_stage + 8 * rows * c, 0, rows, w, stream);
        if (rc) return rc;
    }
    if (C > 1) {
        rc = zkie2_digests_interleave(d_stage, C, rows, d_layers, stream);
    } else {
        rc = (int)cudaMemcpyAsync(d_layers, d_stage, 64 * H, cudaMemcpyDeviceToDevice, stream);
    }
    if (rc) return rc;
    return merkle_build_from_leaves(H, d_layers, stream);
}

// Host-buffer commit: the end-to-end path a drop-in caller of
// CudaDft::dft_batch + CudaMerkleTreeMmcs::commit takes.  Copies the L x w
// coefficient matrix in, runs LDE + tree, and copies back the root and --
// when the pointers are non-null -- the LDE (the tree's leaves) and every
// digest layer.  Synchronous; device buffers come from the stream-ordered
// pool of the current device.
int zkie2_commit_host(const uint64_t* h_coeffs, uint32_t lg_l, uint32_t lg_blowup, uint64_t w,
                      uint64_t* h_lde, uint64_t* h_layers, uint64_t* h_root) {
    if (!h_coeffs || !h_root || w == 0) return (int)cudaErrorInvalidValue;
    DevStreams* st = nullptr;
    int rc = get_streams(&st);
    if (rc) return rc;
    std::lock_guard<std::mutex> call_lock(st->call);
    const uint64_t L = 1ull << lg_l, H = L << lg_blowup;
    const MerkleGeom g = merkle_geometry(H);
    const uint64_t scratch = lde_scratch_elems(lg_l, lg_blowup, w);
    // Pipeline over column blocks: block j is uploaded (copy stream), its LDE
    // computed (compute stream), downloaded (copy_out stream) and absorbed
    // into every row's sponge (hash stream) while block j + 1 is uploaded.
    // Both PCIe directions, the NTT and the hashing overlap; the sponge state
    // of each row waits in HBM between blocks (block boundaries are
    // multiples of 8 columns, i.e. absorption boundaries).  The tree above
    // the leaves follows the last block.
    const uint64_t cw = w >= 64 ? ((w + 3) / 4 + 7) / 8 * 8 : w;  // about four blocks, multiples of 8
    const uint64_t nchunks = (w + cw - 1) / cw;
    uint64_t *d_in = nullptr, *d_lde = nullptr, *d_layers = nullptr, *d_scr = nullptr, *d_states = nullptr;
    cudaStream_t cs = st->compute, hs = st->hash;
    // A failed allocation sets rc; every exit below goes through the frees and
    // the stream synchronisation at the end, so nothing allocated stays behind.
    auto alloc = [&](uint64_t** p, uint64_t bytes) {
        if (!rc) rc = (int)cudaMallocFromPoolAsync((void**)p, bytes, st->pool, cs);
    };
    alloc(&d_in, 8 * L * w);
    alloc(&d_lde, 8 * H * w);
    alloc(&d_layers, 64 * g.total);
    if (scratch) alloc(&d_scr, 8 * scratch);
    if (nchunks > 1) alloc(&d_states, 128 * H);
    if (!rc) rc = p2_ensure_default();
    if (!rc) rc = (int)cudaEventRecord(st->lde_ready, cs);  // the allocations above, in stream order
    if (!rc) rc = (int)cudaStreamWaitEvent(st->copy, st->lde_ready, 0);
    if (!rc) rc = (int)cudaStreamWaitEvent(hs, st->lde_ready, 0);
    for (uint64_t j = 0; !rc && j < nchunks; j++) {
        const uint64_t c0 = j * cw, cn = (w - c0) < cw ? (w - c0) : cw;
        rc = (int)cudaMemcpy2DAsync(d_in + c0, 8 * w, h_coeffs + c0, 8 * w, 8 * cn, L, cudaMemcpyHostToDevice,
                                    st->copy);
        if (!rc) rc = (int)cudaEventRecord(st->in_ready[j], st->copy);
        if (!rc) rc = (int)cudaStreamWaitEvent(cs, st->in_ready[j], 0);
        if (!rc) rc = lde_launch_ld(d_in + c0, d_lde + c0, d_scr ? d_scr + c0 : nullptr, lg_l, lg_blowup, cn, w, cs);
        if (!rc) rc = (int)cudaEventRecord(st->chunk_lde[j], cs);
        if (!rc && h_lde) {
            rc = (int)cudaStreamWaitEvent(st->copy_out, st->chunk_lde[j], 0);
            if (!rc)
                rc = (int)cudaMemcpy2DAsync(h_lde + c0, 8 * w, d_lde + c0, 8 * w, 8 * cn, H, cudaMemcpyDeviceToHost,
                                            st->copy_out);
        }
        if (!rc) rc = (int)cudaStreamWaitEvent(hs, st->chunk_lde[j], 0);
        if (!rc && nchunks > 1)
            rc = launch_leaf_absorb(d_lde, w, c0, cn, H, d_states, d_layers, j == 0, j + 1 == nchunks, hs);
    }
    if (!rc) rc = nchunks > 1 ? merkle_build_from_leaves(H, d_layers, hs) : merkle_build(d_lde, H, w, d_layers, hs);
    if (!rc) {
        if (h_layers)
            rc = (int)cudaMemcpyAsync(h_layers, d_layers, 64 * g.total, cudaMemcpyDeviceToHost, hs);
        else
            rc = (int)cudaMemcpyAsync(h_root, d_layers + 8 * g.offset.back(), 64, cudaMemcpyDeviceToHost, hs);
    }
    // Wait for the side streams (on every path, also after an error part-way)
    // before the buffers they use go back to the pool on the compute stream.
    for (cudaStream_t side : {hs, st->copy_out, st->copy}) {
        cudaError_t e = cudaStreamSynchronize(side);
        if (!rc && e != cudaSuccess) rc = (int)e;
    }
    for (uint64_t* p : {d_in, d_lde, d_layers, d_scr, d_states})
        if (p) cudaFreeAsync(p, cs);
    cudaError_t e = cudaStreamSynchronize(cs);
    if (!rc && e != cudaSuccess) rc = (int)e;
    if (!rc && h_layers)
        for (int i = 0; i < 8; i++) h_root[i] = h_layers[8 * g.offset.back() + i];
    return rc;
}

}  // extern "C"
