// persist.cu -- .fdb files: the reference's on-disk format for IVF-PQ and
// brute-force indexes (host code; the index data moves to and from the
// device through the same paths as fdb_ivfpq_export / fdb_ivfpq_from_trained).
//
// File = 24-byte header + payload (src/persistence/format.rs:76-133,
// mod.rs:169-188):
//   [magic "FORGEDB\0"][version u32 LE][index type u32][flags u32][CRC-32 of payload]
// The payload of an IVF-PQ index is SerializableIVFPQ (ivf_pq.rs:197-262)
// in bincode 1.3's default encoding: little-endian fixed-width integers,
// usize as u64, Vec<T> = u64 length + elements, Option = u8 tag + value,
// unit enum = u32 variant index, struct = its fields in order.  The payload
// of a brute-force index is [metric u8][n u64][dim u64][ids u64 x n]
// [rows f32 x n*dim] (brute_force.rs:277-318).  The CRC is CRC-32/ISO-HDLC
// (crc32fast::hash): reflected polynomial 0xEDB88320, initial value and
// final xor 0xFFFFFFFF.
#include <sys/statvfs.h>
#include <unistd.h>

#include <cerrno>
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>

#include "fdb_device.cuh"
#include "fdb_internal.h"
#include "fdb_kernels.h"

namespace fdb {

// ---------------------------------------------------------------------------
// CRC-32, slicing by 8 (eight derived tables let one step consume 8 bytes)
// ---------------------------------------------------------------------------
struct Crc32Tables {
    uint32_t t[8][256];
    Crc32Tables() {
        for (uint32_t i = 0; i < 256; ++i) {
            uint32_t c = i;
            for (int b = 0; b < 8; ++b) c = (c & 1u) ? (c >> 1) ^ 0xEDB88320u : c >> 1;
            t[0][i] = c;
        }
        for (int k = 1; k < 8; ++k)
            for (uint32_t i = 0; i < 256; ++i) t[k][i] = (t[k - 1][i] >> 8) ^ t[0][t[k - 1][i] & 0xFFu];
    }
};

uint32_t crc32(const uint8_t* p, size_t n) {
    static const Crc32Tables T;
    uint32_t c = 0xFFFFFFFFu;
    while (n >= 8) {
        uint32_t lo, hi;
        std::memcpy(&lo, p, 4);
        std::memcpy(&hi, p + 4, 4);
        lo ^= c;
        c = T.t[7][lo & 0xFFu] ^ T.t[6][(lo >> 8) & 0xFFu] ^ T.t[5][(lo >> 16) & 0xFFu] ^
            T.t[4][lo >> 24] ^ T.t[3][hi & 0xFFu] ^ T.t[2][(hi >> 8) & 0xFFu] ^
            T.t[1][(hi >> 16) & 0xFFu] ^ T.t[0][hi >> 24];
        p += 8;
        n -= 8;
    }
    while (n--) c = T.t[0][(c ^ *p++) & 0xFFu] ^ (c >> 8);
    return c ^ 0xFFFFFFFFu;
}

// ---------------------------------------------------------------------------
// bincode 1.3 (default options) writer / reader
// ---------------------------------------------------------------------------
struct Writer {
    std::vector<uint8_t> b;
    template <typename T>
    void raw(const T* p, size_t n) {
        const size_t o = b.size();
        b.resize(o + n * sizeof(T));
        std::memcpy(b.data() + o, p, n * sizeof(T));
    }
    void u8(uint8_t v) { b.push_back(v); }
    void u32(uint32_t v) { raw(&v, 1); }
    void u64(uint64_t v) { raw(&v, 1); }
    // SerializableVector {id: u64, data: Vec<f32>}
    void vec(uint64_t id, const float* d, size_t n) {
        u64(id);
        u64(n);
        raw(d, n);
    }
};

struct Reader {
    const uint8_t* p;
    size_t n, o = 0;
    template <typename T>
    void raw(T* out, size_t k) {
        if (k > (n - o) / sizeof(T)) fail(FDB_ERR_SERIALIZATION, "io error: unexpected end of file");
        std::memcpy(out, p + o, k * sizeof(T));
        o += k * sizeof(T);
    }
    uint8_t u8() { uint8_t v; raw(&v, 1); return v; }
    uint32_t u32() { uint32_t v; raw(&v, 1); return v; }
    uint64_t u64() { uint64_t v; raw(&v, 1); return v; }
    // a length whose elements of `elem` bytes each must fit in what is left
    uint64_t len(size_t elem) {
        const uint64_t k = u64();
        if (elem && k > (n - o) / elem) fail(FDB_ERR_SERIALIZATION, "io error: unexpected end of file");
        return k;
    }
};

// ---------------------------------------------------------------------------
// header
// ---------------------------------------------------------------------------
static const uint8_t MAGIC[8] = {'F', 'O', 'R', 'G', 'E', 'D', 'B', 0};
constexpr uint32_t FORMAT_VERSION = 1;
constexpr size_t HEADER_SIZE = 24;

struct Header {
    uint32_t version, type, flags, checksum;
};

// verify_header (mod.rs:76-94): size, magic, known type, version, expected
// type, then the payload's CRC.
static Header verify_header(const std::vector<uint8_t>& f, uint32_t expected_type) {
    if (f.size() < HEADER_SIZE) fail(FDB_ERR_INVALID_FORMAT, "invalid file format: file too small for header");
    if (std::memcmp(f.data(), MAGIC, 8) != 0) fail(FDB_ERR_INVALID_FORMAT, "invalid file format: invalid magic bytes");
    Header h;
    std::memcpy(&h.version, f.data() + 8, 4);
    std::memcpy(&h.type, f.data() + 12, 4);
    std::memcpy(&h.flags, f.data() + 16, 4);
    std::memcpy(&h.checksum, f.data() + 20, 4);
    if (h.type < FDB_INDEX_IVFPQ || h.type > FDB_INDEX_BRUTE_FORCE)
        fail(FDB_ERR_INVALID_FORMAT, "invalid file format: unknown index type");
    if (h.version > FORMAT_VERSION)
        fail(FDB_ERR_INVALID_FORMAT, "invalid file format: unsupported version " +
                                         std::to_string(h.version) + " (max supported: 1)");
    if (expected_type && h.type != expected_type)
        fail(FDB_ERR_INVALID_FORMAT, "invalid file format: index type mismatch");
    if (crc32(f.data() + HEADER_SIZE, f.size() - HEADER_SIZE) != h.checksum)
        fail(FDB_ERR_CHECKSUM, "checksum mismatch: file may be corrupted");
    return h;
}

static std::vector<uint8_t> read_file(const char* path) {
    FILE* fp = std::fopen(path, "rb");
    if (!fp) fail(FDB_ERR_IO, std::string("I/O error: cannot open ") + path + ": " + std::strerror(errno));
    std::unique_ptr<FILE, int (*)(FILE*)> guard(fp, std::fclose);
    std::vector<uint8_t> b;
    uint8_t chunk[1 << 16];
    size_t r;
    while ((r = std::fread(chunk, 1, sizeof(chunk), fp)) > 0) b.insert(b.end(), chunk, chunk + r);
    if (std::ferror(fp)) fail(FDB_ERR_IO, std::string("I/O error: read failed: ") + path);
    return b;
}

// check_disk_space (mod.rs:101-165): the directory holding `path` (or the
// working directory) needs the file size plus 10%.  A failed query is not an
// error, as in the reference.
static void check_disk_space(const char* path, uint64_t bytes) {
    const uint64_t need = bytes + bytes / 10;
    std::string dir(path);
    const size_t slash = dir.find_last_of('/');
    dir = slash == std::string::npos ? "." : (slash == 0 ? "/" : dir.substr(0, slash));
    struct statvfs st;
    if (statvfs(dir.c_str(), &st) != 0 && statvfs(".", &st) != 0) return;
    const uint64_t avail = (uint64_t)st.f_bavail * (uint64_t)st.f_frsize;
    if (avail < need)
        fail(FDB_ERR_DISK_SPACE, "insufficient disk space: required " + std::to_string(need) +
                                     " bytes, available " + std::to_string(avail) + " bytes");
}

// write_with_header (mod.rs:169-188)
static void write_with_header(const char* path, uint32_t type, const std::vector<uint8_t>& data) {
    check_disk_space(path, HEADER_SIZE + data.size());
    uint8_t hdr[HEADER_SIZE];
    std::memcpy(hdr, MAGIC, 8);
    const uint32_t v = FORMAT_VERSION, fl = 0, cs = crc32(data.data(), data.size());
    std::memcpy(hdr + 8, &v, 4);
    std::memcpy(hdr + 12, &type, 4);
    std::memcpy(hdr + 16, &fl, 4);
    std::memcpy(hdr + 20, &cs, 4);
    FILE* fp = std::fopen(path, "wb");
    if (!fp) fail(FDB_ERR_IO, std::string("I/O error: cannot create ") + path + ": " + std::strerror(errno));
    bool ok = std::fwrite(hdr, 1, HEADER_SIZE, fp) == HEADER_SIZE &&
              std::fwrite(data.data(), 1, data.size(), fp) == data.size() && std::fflush(fp) == 0 &&
              fsync(fileno(fp)) == 0;
    ok = (std::fclose(fp) == 0) && ok;
    if (!ok) fail(FDB_ERR_IO, std::string("I/O error: write failed: ") + path);
}

// ---------------------------------------------------------------------------
// IVF-PQ payload
// ---------------------------------------------------------------------------
struct IvfParts {
    size_t dim = 0, nlist = 0, m = 0, sub = 0;
    std::vector<float> cents, cb;            // [nlist][dim], [m][256][sub]
    std::vector<uint64_t> cent_ids, cb_ids;  // [nlist], [m*256]
    std::vector<uint64_t> offs, ids;         // [nlist+1], [n]
    std::vector<uint8_t> codes;              // [n][m]
    uint64_t nprobe = 1;
    uint32_t metric = 0;
    bool has_rr = false;
    std::vector<uint64_t> rr_ids;
    std::vector<float> rr_x;
    uint64_t rerank_factor = 1;
};

static std::vector<uint8_t> encode_ivf(const IvfParts& P) {
    Writer w;
    const size_t n = P.ids.size();
    w.b.reserve(64 + P.nlist * (16 + P.dim * 4) + P.m * KSUB * (16 + P.sub * 4) +
                P.nlist * 16 + n * (16 + P.m) + P.rr_ids.size() * (16 + P.dim * 4));
    w.u64(P.nlist);  // centroids
    for (size_t l = 0; l < P.nlist; ++l) w.vec(P.cent_ids[l], P.cents.data() + l * P.dim, P.dim);
    w.u64(P.m);  // pq.codebooks
    for (size_t s = 0; s < P.m; ++s) {
        w.u64(KSUB);
        for (size_t j = 0; j < (size_t)KSUB; ++j)
            w.vec(P.cb_ids[s * KSUB + j], P.cb.data() + (s * KSUB + j) * P.sub, P.sub);
    }
    w.u64(P.m);    // pq.n_subvectors
    w.u64(P.sub);  // pq.subvector_dim
    w.u64(P.dim);  // pq.dim
    w.u64(P.nlist);  // partitions
    for (size_t l = 0; l < P.nlist; ++l) {
        const uint64_t b = P.offs[l], e = P.offs[l + 1];
        w.u64(e - b);
        w.raw(P.ids.data() + b, e - b);
        w.u64(e - b);
        for (uint64_t r = b; r < e; ++r) {
            w.u64(P.m);
            w.raw(P.codes.data() + r * P.m, P.m);
        }
    }
    w.u64(P.nprobe);
    w.u32(P.metric);
    w.u8(P.has_rr ? 1 : 0);
    if (P.has_rr) {
        w.u64(P.rr_ids.size());
        for (size_t i = 0; i < P.rr_ids.size(); ++i)
            w.vec(P.rr_ids[i], P.rr_x.data() + i * P.dim, P.dim);
    }
    w.u64(P.rerank_factor);
    return std::move(w.b);
}

// Parses SerializableIVFPQ and checks what the engine relies on (the
// reference would panic later on most of these).
static IvfParts decode_ivf(const uint8_t* p, size_t n) {
    Reader r{p, n};
    IvfParts P;
    auto bad = [](const std::string& m) { fail(FDB_ERR_INVALID_FORMAT, "invalid file format: " + m); };
    const uint64_t nlist = r.len(16);
    P.nlist = nlist;
    P.cent_ids.resize(nlist);
    for (uint64_t l = 0; l < nlist; ++l) {
        P.cent_ids[l] = r.u64();
        const uint64_t d = r.len(4);
        if (l == 0) {
            P.dim = d;
            P.cents.resize(nlist * d);
        } else if (d != P.dim) {
            bad("centroids of different dimensions");
        }
        r.raw(P.cents.data() + l * d, d);
    }
    const uint64_t ncb = r.len(8);
    std::vector<std::vector<uint64_t>> cbid(ncb);
    std::vector<std::vector<float>> cbx(ncb);
    uint64_t sub = 0;
    for (uint64_t s = 0; s < ncb; ++s) {
        const uint64_t ne = r.len(16);
        for (uint64_t j = 0; j < ne; ++j) {
            cbid[s].push_back(r.u64());
            const uint64_t d = r.len(4);
            if (s == 0 && j == 0) sub = d;
            else if (d != sub) bad("codebook entries of different lengths");
            const size_t o = cbx[s].size();
            cbx[s].resize(o + d);
            r.raw(cbx[s].data() + o, d);
        }
    }
    const uint64_t nsv = r.u64(), sdim = r.u64(), pdim = r.u64();
    const uint64_t npart = r.len(16);
    std::vector<uint64_t> sizes(npart);
    P.offs.assign(npart + 1, 0);
    for (uint64_t l = 0; l < npart; ++l) {
        const uint64_t ni = r.len(8);
        const size_t o = P.ids.size();
        P.ids.resize(o + ni);
        r.raw(P.ids.data() + o, ni);
        const uint64_t nc = r.len(8);
        if (nc != ni) bad("partition with different numbers of ids and codes");
        if (l == 0 && nsv > (uint64_t)1 << 20) bad("n_subvectors out of range");
        P.codes.resize(P.codes.size() + nc * nsv);
        for (uint64_t j = 0; j < nc; ++j) {
            const uint64_t cl = r.len(1);
            if (cl != nsv) bad("code length differs from n_subvectors");
            r.raw(P.codes.data() + (o + j) * nsv, cl);
        }
        P.offs[l + 1] = P.ids.size();
    }
    P.nprobe = r.u64();
    P.metric = r.u32();
    if (P.metric > 4) fail(FDB_ERR_SERIALIZATION, "invalid value: unknown DistanceMetric variant");
    const uint8_t tag = r.u8();
    if (tag > 1) fail(FDB_ERR_SERIALIZATION, "invalid value: Option tag");
    P.has_rr = tag == 1;
    if (P.has_rr) {
        const uint64_t nv = r.len(16);
        P.rr_ids.resize(nv);
        for (uint64_t i = 0; i < nv; ++i) {
            P.rr_ids[i] = r.u64();
            const uint64_t d = r.len(4);
            if (d != pdim) bad("original vector of a different dimension");
            const size_t o = P.rr_x.size();
            P.rr_x.resize(o + d);
            r.raw(P.rr_x.data() + o, d);
        }
    }
    P.rerank_factor = r.u64();
    // shape checks
    if (nlist == 0) bad("no centroids");
    if (P.dim != pdim) bad("centroid dimension differs from the quantizer's");
    if (ncb != nsv || nsv == 0 || sdim == 0 || nsv * sdim != pdim || sub != sdim)
        bad("quantizer shape inconsistent");
    if (npart != nlist) bad("partition count differs from centroid count");
    for (uint64_t s = 0; s < ncb; ++s)
        if (cbid[s].size() != (size_t)KSUB)
            fail(FDB_ERR_UNSUPPORTED, "operation not supported: codebooks with fewer than 256 entries");
    P.m = nsv;
    P.sub = sdim;
    P.cb.resize(nsv * KSUB * sdim);
    P.cb_ids.resize(nsv * KSUB);
    for (uint64_t s = 0; s < ncb; ++s) {
        std::copy(cbx[s].begin(), cbx[s].end(), P.cb.begin() + s * KSUB * sdim);
        std::copy(cbid[s].begin(), cbid[s].end(), P.cb_ids.begin() + s * KSUB);
    }
    return P;
}

static IvfParts gather_ivf(fdb_ivfpq* h) {
    FDB_REQUIRE(h->shard_world <= 1, FDB_ERR_UNSUPPORTED,
                "operation not supported: saving a sharded index");
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    IvfParts P;
    P.dim = h->dim;
    P.nlist = h->nlist;
    P.m = h->m;
    P.sub = h->dim / h->m;
    P.cents.resize(h->nlist * h->dim);
    P.cb.resize(h->m * KSUB * P.sub);
    P.codes.resize(h->n_total * h->m);
    FDB_CUDA(cudaMemcpyAsync(P.cents.data(), h->cents.p, P.cents.size() * 4, cudaMemcpyDeviceToHost, s));
    FDB_CUDA(cudaMemcpyAsync(P.cb.data(), h->cb.p, P.cb.size() * 4, cudaMemcpyDeviceToHost, s));
    if (h->n_total)
        FDB_CUDA(cudaMemcpyAsync(P.codes.data(), h->codes.p, P.codes.size(), cudaMemcpyDeviceToHost, s));
    FDB_CUDA(cudaStreamSynchronize(s));
    P.cent_ids = h->cent_ids;
    P.cb_ids = h->cb_ids;
    P.offs = h->h_offs_full;
    P.ids = h->h_ids;
    P.nprobe = h->nprobe.load(std::memory_order_relaxed);
    P.metric = (uint32_t)h->metric;
    P.has_rr = h->rerank;
    if (h->rerank) {
        P.rr_ids = h->rr_ids;
        P.rr_x = h->rr_x;
    }
    P.rerank_factor = h->rerank_factor;
    return P;
}

void ivfpq_save(fdb_ivfpq* h, const char* path) {
    const IvfParts P = gather_ivf(h);
    write_with_header(path, FDB_INDEX_IVFPQ, encode_ivf(P));
}

// from_serializable (ivf_pq.rs:1917-1942) onto the device.
void ivfpq_load_file(fdb_ivfpq* h, const char* path) {
    const std::vector<uint8_t> f = read_file(path);
    verify_header(f, FDB_INDEX_IVFPQ);
    const IvfParts P = decode_ivf(f.data() + HEADER_SIZE, f.size() - HEADER_SIZE);
    // (codes need no range check: every byte names one of the 256 entries)
    h->dim = P.dim;
    h->nlist = P.nlist;
    h->m = P.m;
    h->metric = (int)P.metric;
    h->cent_ids = P.cent_ids;
    h->cb_ids = P.cb_ids;
    ivfpq_load(h, P.cents.data(), P.cb.data(), P.offs.data(), P.ids.data(), P.codes.data());
    h->nprobe.store(P.nprobe, std::memory_order_relaxed);  // stored as read, not clamped
    if (P.has_rr) ivfpq_enable_reranking(h, P.rr_x.data(), P.rr_ids.data(), P.rr_ids.size(), 1);
    h->rerank_factor = P.rerank_factor;
}

// ---------------------------------------------------------------------------
// brute force payload
// ---------------------------------------------------------------------------
void bf_save(fdb_bf* h, const char* path) {
    const size_t n = h->h_ids.size(), dim = n ? h->dim : 0;
    Writer w;
    w.b.reserve(17 + n * 8 + n * dim * 4);
    w.u8((uint8_t)h->metric);
    w.u64(n);
    w.u64(dim);
    w.raw(h->h_ids.data(), n);
    w.raw(h->h_x.data(), n * dim);
    write_with_header(path, FDB_INDEX_BRUTE_FORCE, w.b);
}

struct BfParts {
    uint8_t metric;
    uint64_t n, dim;
    const uint8_t* ids;
    const uint8_t* rows;
};

static BfParts decode_bf(const uint8_t* p, size_t len) {
    if (len < 17) fail(FDB_ERR_INVALID_FORMAT, "invalid file format: brute-force payload too small");
    BfParts b;
    b.metric = p[0];
    if (b.metric > 4) fail(FDB_ERR_INVALID_FORMAT, "invalid file format: unknown metric byte");
    std::memcpy(&b.n, p + 1, 8);
    std::memcpy(&b.dim, p + 9, 8);
    // 17 + n*8 + n*dim*4 bytes at least (trailing bytes are allowed)
    const uint64_t room = len - 17;
    if (b.n > room / 8 || (b.n && b.dim > (room - b.n * 8) / 4 / b.n))
        fail(FDB_ERR_INVALID_FORMAT, "invalid file format: brute-force payload truncated");
    b.ids = p + 17;
    b.rows = p + 17 + b.n * 8;
    return b;
}

void bf_load_file(fdb_bf* h, const char* path) {
    const std::vector<uint8_t> f = read_file(path);
    verify_header(f, FDB_INDEX_BRUTE_FORCE);
    const BfParts b = decode_bf(f.data() + HEADER_SIZE, f.size() - HEADER_SIZE);
    h->metric = b.metric;
    h->dim = b.dim;
    h->h_ids.resize(b.n);
    h->h_x.resize(b.n * b.dim);
    std::memcpy(h->h_ids.data(), b.ids, b.n * 8);
    std::memcpy(h->h_x.data(), b.rows, b.n * b.dim * 4);
    h->row0 = 0;
    h->n = b.n;
    h->dirty = true;
}

void file_inspect(const char* path, fdb_file_info* info) {
    const std::vector<uint8_t> f = read_file(path);
    const Header hd = verify_header(f, 0);
    std::memset(info, 0, sizeof(*info));
    info->version = hd.version;
    info->index_type = hd.type;
    info->flags = hd.flags;
    info->checksum = hd.checksum;
    const uint8_t* p = f.data() + HEADER_SIZE;
    const size_t n = f.size() - HEADER_SIZE;
    if (hd.type == FDB_INDEX_IVFPQ) {
        const IvfParts P = decode_ivf(p, n);
        info->n = P.ids.size();
        info->dim = P.dim;
        info->nlist = P.nlist;
        info->m = P.m;
        info->nprobe = P.nprobe;
        info->metric = (int32_t)P.metric;
        info->has_rerank = P.has_rr;
        info->n_rerank = P.rr_ids.size();
        info->rerank_factor = P.rerank_factor;
    } else if (hd.type == FDB_INDEX_BRUTE_FORCE) {
        const BfParts b = decode_bf(p, n);
        info->n = b.n;
        info->dim = b.dim;
        info->metric = b.metric;
    }
}

}  // namespace fdb
