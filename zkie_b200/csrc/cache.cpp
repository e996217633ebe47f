// cache.cpp -- the ZKIEBCH2 weight-cache file, written from and read back into
// device buffers.
//
// Layout (the reference writes it in three pieces):
//   1. header = bincode 1.3.3 (default options: little-endian, fixed-width
//      integers, u64 lengths) of (b"ZKIEBCH2", BatchCacheMetadata, Commitment)
//      (crates/zkie-core/src/pcs/cache.rs:7-70).  BatchCacheMetadata:
//      schema_version u32 (2), model_id String, group_id String, table_ids
//      Vec<String>, table_arity u32, num_tables u32, security_level u32,
//      pow_bits u32, source_digest [u8; 32]; Commitment = MerkleCap: a
//      Vec<[F; 8]> of one digest (cap height 0), F as its u64 word;
//   2. the committed matrices (Whir::serialize_batch_prover_data_into,
//      pcs/whir.rs:542-559): u64 count, then per matrix u64 width, u64 value
//      count and the values as little-endian u64;
//   3. the digest layers (vendor/p3-merkle-tree/src/merkle_tree.rs:224-244,
//      write_digest_layers): u64 layer count, u64 length of each layer, u64
//      arity of each step (2 for the binary tree), then every layer's digests
//      (8 little-endian u64 each).
// Pieces 2 and 3 live in HBM after a commit (the LDE is the committed matrix,
// the flat digest-layer buffer holds every layer), so they stream between the
// device and the file through two pinned staging buffers: the copy of one
// chunk overlaps the file I/O of the other.
#include <fcntl.h>
#include <unistd.h>

#include <cstring>
#include <vector>

#include "../../include/zkie2.h"
#include "common.cuh"
#include "internal.h"

namespace zk {
namespace {

constexpr uint64_t kStage = 32ull << 20;  // bytes per staging buffer
constexpr char kMagic[8] = {'Z', 'K', 'I', 'E', 'B', 'C', 'H', '2'};

struct ByteSink {
    uint8_t* out;
    uint64_t cap, len = 0;
    void put(const void* p, uint64_t n) {
        if (len + n <= cap && out) std::memcpy(out + len, p, n);
        len += n;
    }
    void u32(uint32_t v) { put(&v, 4); }
    void u64(uint64_t v) { put(&v, 8); }
    void str(const char* s) {
        const uint64_t n = std::strlen(s);
        u64(n);
        put(s, n);
    }
};

bool write_all(int fd, const void* p, uint64_t n) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    while (n) {
        const ssize_t w = ::write(fd, b, n > (1ull << 30) ? (1ull << 30) : n);
        if (w <= 0) return false;
        b += w;
        n -= (uint64_t)w;
    }
    return true;
}

bool read_all(int fd, void* p, uint64_t n) {
    uint8_t* b = static_cast<uint8_t*>(p);
    while (n) {
        const ssize_t r = ::read(fd, b, n > (1ull << 30) ? (1ull << 30) : n);
        if (r <= 0) return false;
        b += r;
        n -= (uint64_t)r;
    }
    return true;
}

// Pinned double buffer with one event per half.
struct Staging {
    uint8_t* buf[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    int init() {
        for (int i = 0; i < 2; i++) {
            ZK_TRY(cudaMallocHost((void**)&buf[i], kStage));
            ZK_TRY(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming));
        }
        return 0;
    }
    ~Staging() {
        for (int i = 0; i < 2; i++) {
            if (ev[i]) cudaEventDestroy(ev[i]);
            if (buf[i]) cudaFreeHost(buf[i]);
        }
    }
};

// Device bytes -> file, chunk i + 1 copied while chunk i is written.
int stream_out(int fd, const uint8_t* d, uint64_t n, Staging& st, cudaStream_t s) {
    const uint64_t chunks = ceil_div(n, kStage);
    auto issue = [&](uint64_t c) -> int {
        const uint64_t off = c * kStage, len = n - off < kStage ? n - off : kStage;
        ZK_TRY(cudaMemcpyAsync(st.buf[c & 1], d + off, len, cudaMemcpyDeviceToHost, s));
        ZK_TRY(cudaEventRecord(st.ev[c & 1], s));
        return 0;
    };
    if (chunks) {
        int rc = issue(0);
        if (rc) return rc;
    }
    for (uint64_t c = 0; c < chunks; c++) {
        ZK_TRY(cudaEventSynchronize(st.ev[c & 1]));
        if (c + 1 < chunks) {
            const int rc = issue(c + 1);
            if (rc) return rc;
        }
        const uint64_t off = c * kStage, len = n - off < kStage ? n - off : kStage;
        if (!write_all(fd, st.buf[c & 1], len)) return (int)cudaErrorUnknown;
    }
    return 0;
}

// File -> device bytes, chunk i + 1 read while chunk i is copied.
int stream_in(int fd, uint8_t* d, uint64_t n, Staging& st, cudaStream_t s) {
    const uint64_t chunks = ceil_div(n, kStage);
    bool pending[2] = {false, false};
    for (uint64_t c = 0; c < chunks; c++) {
        const int b = (int)(c & 1);
        if (pending[b]) ZK_TRY(cudaEventSynchronize(st.ev[b]));  // the buffer's previous copy is done
        const uint64_t off = c * kStage, len = n - off < kStage ? n - off : kStage;
        if (!read_all(fd, st.buf[b], len)) return (int)cudaErrorInvalidValue;
        ZK_TRY(cudaMemcpyAsync(d + off, st.buf[b], len, cudaMemcpyHostToDevice, s));
        ZK_TRY(cudaEventRecord(st.ev[b], s));
        pending[b] = true;
    }
    return (int)cudaStreamSynchronize(s);
}

}  // namespace
}  // namespace zk

using namespace zk;

extern "C" {

uint64_t zkie2_cache_header(const char* model_id, const char* group_id, const char* const* table_ids,
                            uint32_t num_tables, uint32_t table_arity, uint32_t security_level, uint32_t pow_bits,
                            const uint8_t* source_digest, const uint64_t* root, uint8_t* out, uint64_t out_cap) {
    if (!model_id || !group_id || (num_tables && !table_ids) || !source_digest || !root) return 0;
    ByteSink b{out, out_cap};
    b.put(kMagic, 8);
    b.u32(2);  // BATCH_CACHE_SCHEMA_VERSION
    b.str(model_id);
    b.str(group_id);
    b.u64(num_tables);
    for (uint32_t i = 0; i < num_tables; i++) {
        if (!table_ids[i]) return 0;
        b.str(table_ids[i]);
    }
    b.u32(table_arity);
    b.u32(num_tables);
    b.u32(security_level);
    b.u32(pow_bits);
    b.put(source_digest, 32);
    b.u64(1);  // MerkleCap of cap height 0: one digest
    for (int i = 0; i < 8; i++) b.u64(root[i]);
    return b.len;
}

int zkie2_cache_write(const char* path, const uint8_t* header, uint64_t header_len, const uint64_t* d_lde,
                      uint64_t rows, uint64_t width, const uint64_t* d_layers, cudaStream_t stream) {
    if (!path || !header || !header_len || !d_lde || !d_layers || !rows || !width) return (int)cudaErrorInvalidValue;
    const MerkleGeom g = merkle_geometry(rows);
    const int fd = ::open(path, O_WRONLY | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) return (int)cudaErrorInvalidValue;
    Staging st;
    int rc = st.init();
    std::vector<uint64_t> words = {1, width, rows * width};
    if (!rc && !(write_all(fd, header, header_len) && write_all(fd, words.data(), 8 * words.size())))
        rc = (int)cudaErrorUnknown;
    if (!rc) rc = stream_out(fd, reinterpret_cast<const uint8_t*>(d_lde), 8 * rows * width, st, stream);
    if (!rc) {
        words.clear();
        words.push_back(g.len.size());
        for (uint64_t l : g.len) words.push_back(l);
        for (size_t i = 0; i + 1 < g.len.size(); i++) words.push_back(2);
        if (!write_all(fd, words.data(), 8 * words.size())) rc = (int)cudaErrorUnknown;
    }
    if (!rc) rc = stream_out(fd, reinterpret_cast<const uint8_t*>(d_layers), 64 * g.total, st, stream);
    cudaStreamSynchronize(stream);  // no copy into the staging buffers outlives them
    if (::close(fd) != 0 && !rc) rc = (int)cudaErrorUnknown;
    return rc;
}

int zkie2_cache_read(const char* path, uint64_t header_len, uint64_t rows, uint64_t width, uint64_t* d_lde,
                     uint64_t* d_layers, cudaStream_t stream) {
    if (!path || !d_lde || !d_layers || !rows || !width) return (int)cudaErrorInvalidValue;
    const MerkleGeom g = merkle_geometry(rows);
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) return (int)cudaErrorInvalidValue;
    int rc = 0;
    if (::lseek(fd, (off_t)header_len, SEEK_SET) != (off_t)header_len) rc = (int)cudaErrorInvalidValue;
    uint64_t m[3] = {0, 0, 0};
    if (!rc && !read_all(fd, m, 24)) rc = (int)cudaErrorInvalidValue;
    if (!rc && (m[0] != 1 || m[1] != width || m[2] != rows * width)) rc = (int)cudaErrorInvalidValue;
    Staging st;
    if (!rc) rc = st.init();
    if (!rc) rc = stream_in(fd, reinterpret_cast<uint8_t*>(d_lde), 8 * rows * width, st, stream);
    const uint64_t nl = g.len.size();
    std::vector<uint64_t> words(1 + nl + (nl ? nl - 1 : 0));
    if (!rc && !read_all(fd, words.data(), 8 * words.size())) rc = (int)cudaErrorInvalidValue;
    if (!rc && words[0] != nl) rc = (int)cudaErrorInvalidValue;
    for (uint64_t i = 0; !rc && i < nl; i++)
        if (words[1 + i] != g.len[i]) rc = (int)cudaErrorInvalidValue;
    for (uint64_t i = 0; !rc && i + 1 < nl; i++)
        if (words[1 + nl + i] != 2) rc = (int)cudaErrorInvalidValue;
    if (!rc) rc = stream_in(fd, reinterpret_cast<uint8_t*>(d_layers), 64 * g.total, st, stream);
    cudaStreamSynchronize(stream);  // no copy out of the staging buffers outlives them
    ::close(fd);
    return rc;
}

}  // extern "C"
