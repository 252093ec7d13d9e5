// Sidecar loader, process-wide tensor registry and the reference's operator
// surface keyed by ggml tensor name.  Host code only.
//
// Byte layout of the sidecar (unchanged from source/q4rdna.cu:26-50 and the
// writers source/q4rdna_sidecar_pack.cpp:23-47, source/pack_q4rdna_sidecar.py:16-23):
//   header 48 B: magic "Q4RDNA1\0", u32 version=1, count, group=64,
//                tile_rows=32, tile_bytes=1088, reserved, u64 data_offset, data_bytes
//   count entries of 96 B: char name[64], u32 rows, columns, u64 offset
//                (absolute), size, reserved
//   data region at data_offset (4096-aligned by both writers), tensors 256-aligned.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "q4rdna.h"
#include "q4rdna_tile.h"

namespace {

#pragma pack(push, 1)
struct FileHeader {
    char magic[8];
    uint32_t version, count, group, tile_rows, tile_bytes, reserved;
    uint64_t data_offset, data_bytes;
};
struct FileEntry {
    char name[64];
    uint32_t rows, columns;
    uint64_t offset, size, reserved;
};
#pragma pack(pop)
static_assert(sizeof(FileHeader) == 48, "sidecar header is 48 bytes");
static_assert(sizeof(FileEntry) == 96, "sidecar entry is 96 bytes");

struct Entry {
    std::string name;
    uint32_t rows = 0, cols = 0;
    uint64_t rel = 0, size = 0;
    std::unique_ptr<std::atomic<uint64_t>> hits{new std::atomic<uint64_t>(0)};
};

struct FileCloser {
    void operator()(FILE *f) const { if (f) std::fclose(f); }
};

}  // namespace

struct q4rdna_sidecar {
    int device = -1;
    uint8_t *data = nullptr;
    uint64_t data_bytes = 0;
    std::vector<Entry> entries;
    std::unordered_map<std::string, size_t> index;
};

namespace {

bool read_exact(FILE *f, void *dst, size_t n) { return std::fread(dst, 1, n, f) == n; }

// Validation rules of source/q4rdna.cu:131-152, plus the 16-byte tensor
// alignment the 128-bit loads need (both reference writers align to 256).
q4rdna_status parse(FILE *f, FileHeader &h, std::vector<FileEntry> &es) {
    if (!read_exact(f, &h, sizeof(h))) return Q4RDNA_ERR_IO;
    if (std::memcmp(h.magic, "Q4RDNA1", 8) != 0 || h.version != 1 || h.group != Q4_GROUP ||
        h.tile_rows != Q4_TILE_ROWS || h.tile_bytes != Q4_TILE_BYTES)
        return Q4RDNA_ERR_FORMAT;
    if (h.count > (1u << 24)) return Q4RDNA_ERR_FORMAT;
    es.resize(h.count);
    if (h.count && !read_exact(f, es.data(), es.size() * sizeof(FileEntry))) return Q4RDNA_ERR_IO;
    if (h.data_offset + h.data_bytes < h.data_offset) return Q4RDNA_ERR_FORMAT;
    for (const FileEntry &e : es) {
        if (std::memchr(e.name, '\0', sizeof(e.name)) == nullptr || e.offset < h.data_offset ||
            e.offset + e.size < e.offset || e.offset + e.size > h.data_offset + h.data_bytes ||
            e.rows % Q4_TILE_ROWS != 0 || e.columns % Q4_GROUP != 0 ||
            e.size != Q4_TENSOR_BYTES(e.rows, e.columns) || ((e.offset - h.data_offset) & 15u) != 0 ||
            e.rows == 0 || e.columns == 0 || e.rows > 0x7fffffffu || e.columns > 0x7fffffffu)
            return Q4RDNA_ERR_FORMAT;
    }
    return Q4RDNA_OK;
}

}  // namespace

extern "C" {

q4rdna_status q4rdna_sidecar_open(const char *path, int device, q4rdna_sidecar **out) {
    if (path == nullptr || out == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    std::unique_ptr<FILE, FileCloser> f(std::fopen(path, "rb"));
    if (!f) return Q4RDNA_ERR_IO;
    FileHeader h{};
    std::vector<FileEntry> es;
    q4rdna_status st = parse(f.get(), h, es);
    if (st != Q4RDNA_OK) return st;
    // The data region must be fully present before any device memory is taken.
    if (std::fseek(f.get(), 0, SEEK_END) != 0) return Q4RDNA_ERR_IO;
    const long end = std::ftell(f.get());
    if (end < 0 || (uint64_t)end < h.data_offset + h.data_bytes) return Q4RDNA_ERR_IO;

    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return Q4RDNA_ERR_DEVICE;
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return Q4RDNA_ERR_DEVICE;

    std::unique_ptr<q4rdna_sidecar> sc(new q4rdna_sidecar());
    sc->device = device;
    sc->data_bytes = h.data_bytes;
    st = Q4RDNA_OK;
    if (h.data_bytes && cudaMalloc(&sc->data, h.data_bytes) != cudaSuccess) st = Q4RDNA_ERR_CUDA;
    if (st == Q4RDNA_OK && h.data_bytes) {
        // 64 MiB chunks through a pinned staging buffer (source/q4rdna.cu:159-174).
        const size_t chunk = 64u << 20;
        void *stage = nullptr;
        if (cudaMallocHost(&stage, chunk) != cudaSuccess) st = Q4RDNA_ERR_CUDA;
        if (st == Q4RDNA_OK && std::fseek(f.get(), (long)h.data_offset, SEEK_SET) != 0) st = Q4RDNA_ERR_IO;
        for (uint64_t done = 0; st == Q4RDNA_OK && done < h.data_bytes;) {
            const size_t n = (size_t)std::min<uint64_t>(chunk, h.data_bytes - done);
            if (!read_exact(f.get(), stage, n)) { st = Q4RDNA_ERR_IO; break; }
            if (cudaMemcpy(sc->data + done, stage, n, cudaMemcpyHostToDevice) != cudaSuccess) { st = Q4RDNA_ERR_CUDA; break; }
            done += n;
        }
        if (stage) cudaFreeHost(stage);
    }
    if (st != Q4RDNA_OK) {
        if (sc->data) cudaFree(sc->data);
        cudaSetDevice(prev);
        return st;
    }
    sc->entries.resize(es.size());
    for (size_t i = 0; i < es.size(); ++i) {
        Entry &e = sc->entries[i];
        e.name = es[i].name;
        e.rows = es[i].rows;
        e.cols = es[i].columns;
        e.rel = es[i].offset - h.data_offset;
        e.size = es[i].size;
        sc->index.emplace(e.name, i);  // first entry of a duplicated name wins
    }
    cudaSetDevice(prev);
    *out = sc.release();
    return Q4RDNA_OK;
}

void q4rdna_sidecar_close(q4rdna_sidecar *sc) {
    if (sc == nullptr) return;
    if (sc->data) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(sc->device);
        cudaFree(sc->data);
        cudaSetDevice(prev);
    }
    delete sc;
}

int q4rdna_sidecar_count(const q4rdna_sidecar *sc) { return sc ? (int)sc->entries.size() : 0; }

q4rdna_status q4rdna_sidecar_entry(const q4rdna_sidecar *sc, int i, char name_out[64], int *rows, int *cols,
                                   uint64_t *rel) {
    if (sc == nullptr || i < 0 || i >= (int)sc->entries.size()) return Q4RDNA_ERR_INVALID_ARGUMENT;
    const Entry &e = sc->entries[i];
    if (name_out) {
        std::memset(name_out, 0, 64);
        std::memcpy(name_out, e.name.data(), std::min<size_t>(63, e.name.size()));
    }
    if (rows) *rows = (int)e.rows;
    if (cols) *cols = (int)e.cols;
    if (rel) *rel = e.rel;
    return Q4RDNA_OK;
}

q4rdna_status q4rdna_sidecar_find(const q4rdna_sidecar *sc, const char *name, int *rows, int *cols,
                                  const uint8_t **tiles) {
    if (sc == nullptr || name == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    const auto it = sc->index.find(name);
    if (it == sc->index.end()) return Q4RDNA_ERR_NOT_FOUND;
    const Entry &e = sc->entries[it->second];
    if (rows) *rows = (int)e.rows;
    if (cols) *cols = (int)e.cols;
    if (tiles) *tiles = sc->data + e.rel;
    return Q4RDNA_OK;
}

}  // extern "C"

// ------------------------------------------- process registry (ggml surface)
namespace {

struct Registry {
    std::mutex mu;
    bool attempted = false;       // load tried (the reference's call_once, q4rdna.cu:698)
    q4rdna_sidecar *sc = nullptr; // null: disabled
    size_t ws_bytes = 0;          // per-stream split-K workspace size
    std::map<cudaStream_t, void *> ws;
};

Registry &registry() {
    // Process lifetime, like the reference (q4rdna.cu:67-71).
    static Registry *r = new Registry();
    return *r;
}

std::atomic<uint64_t> g_op_launches{0};
std::atomic<bool> g_atexit{false};

const char *sidecar_path() {
    const char *p = std::getenv("LLAMA_Q4_RDNA_SIDECAR");
    return (p == nullptr || p[0] == '\0') ? nullptr : p;
}

// LLAMA_Q4_RDNA_SCOPE name filter, source/q4rdna.cu:685-696.
bool in_scope(const char *name) {
    const char *scope = std::getenv("LLAMA_Q4_RDNA_SCOPE");
    if (scope == nullptr) return true;
    if (std::strcmp(scope, "ffn") == 0 && std::strstr(name, ".ffn_") == nullptr) return false;
    if (std::strcmp(scope, "qkv-fallback") == 0 &&
        (std::strstr(name, ".attn_q.") || std::strstr(name, ".attn_k.") || std::strstr(name, ".attn_v.")))
        return false;
    if (std::strcmp(scope, "hotspot") == 0 && std::strstr(name, ".ffn_gate.") == nullptr &&
        std::strstr(name, ".ffn_up.") == nullptr)
        return false;
    if (std::strcmp(scope, "attn") == 0 && std::strstr(name, ".attn_") == nullptr) return false;
    return true;
}

void *stream_workspace(Registry &r, cudaStream_t stream);

// Loads on first use onto the current device; null if disabled.  The split-K
// workspace of the calling stream is allocated in the same one-time load, next
// to the weights, so later hook calls on that stream allocate nothing.
q4rdna_sidecar *ensure_loaded(Registry &r, cudaStream_t stream) {
    if (r.attempted) return r.sc;
    r.attempted = true;
    const char *path = sidecar_path();
    if (path == nullptr) return nullptr;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    q4rdna_sidecar *sc = nullptr;
    const q4rdna_status st = q4rdna_sidecar_open(path, dev, &sc);
    if (st != Q4RDNA_OK) {
        std::fprintf(stderr, "Q4_RDNA: cannot load sidecar %s: %s\n", path, q4rdna_status_string(st));
        return nullptr;
    }
    size_t ws = 0;
    for (const Entry &e : sc->entries)
        for (int op = Q4RDNA_OP_PLAIN; op <= Q4RDNA_OP_SWIGLU; ++op)
            ws = std::max(ws, q4rdna_workspace_bytes((int)e.rows, (int)e.cols, 1, op, nullptr));
    r.ws_bytes = ws;
    r.sc = sc;
    if (ws > 0 && stream_workspace(r, stream) == nullptr) {
        std::fprintf(stderr, "Q4_RDNA: cannot allocate the %zu-byte split-K workspace\n", ws);
        q4rdna_sidecar_close(sc);
        r.sc = nullptr;
        return nullptr;
    }
    if (!g_atexit.exchange(true)) std::atexit(q4rdna_report_stats);
    std::fprintf(stderr, "Q4_RDNA: loaded %d tensors, %.2f GiB on device %d from %s\n", (int)sc->entries.size(),
                 double(sc->data_bytes) / (1024.0 * 1024.0 * 1024.0), dev, path);
    return sc;
}

// Workspace of one stream: the loading stream's comes with the load; any other
// stream's is allocated and zeroed on its first call (so the first call on a
// stream must not be inside a graph capture).  All are freed by
// q4rdna_registry_reset.
void *stream_workspace(Registry &r, cudaStream_t stream) {
    if (r.ws_bytes == 0) return nullptr;
    auto it = r.ws.find(stream);
    if (it != r.ws.end()) return it->second;
    void *p = nullptr;
    if (cudaMalloc(&p, r.ws_bytes) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, r.ws_bytes) != cudaSuccess) { cudaFree(p); return nullptr; }
    r.ws.emplace(stream, p);
    return p;
}

struct Found {
    const uint8_t *tiles = nullptr;
    const Entry *entry = nullptr;
};

// q4rdna_find (source/q4rdna.cu:682-705): scope, lazy load, device, name, shape.
bool find(Registry &r, const char *name, int64_t ne0, int64_t ne1, cudaStream_t stream, Found &out) {
    if (name == nullptr || sidecar_path() == nullptr || !in_scope(name)) return false;
    q4rdna_sidecar *sc = ensure_loaded(r, stream);
    if (sc == nullptr) return false;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != sc->device) return false;
    const auto it = sc->index.find(name);
    if (it == sc->index.end()) return false;
    const Entry &e = sc->entries[it->second];
    if (ne0 != (int64_t)e.cols || ne1 != (int64_t)e.rows) return false;
    out.tiles = sc->data + e.rel;
    out.entry = &e;
    return true;
}

}  // namespace

void noalloc_forget_devices();  // q4rdna_noalloc.cu

namespace {
// Launch options of the hooks: the sidecar's tiles are written once at load and
// never again, so each GEMV may start streaming them while the previous kernel
// on the stream finishes (Q4RDNA_CFG_OVERLAP_PREVIOUS).  LLAMA_Q4_RDNA_OVERLAP=0
// turns that off.
const q4rdna_cfg *hook_cfg() {
    static const q4rdna_cfg c = [] {
        q4rdna_cfg v{};
        const char *e = std::getenv("LLAMA_Q4_RDNA_OVERLAP");
        v.flags = (e != nullptr && std::strcmp(e, "0") == 0) ? 0 : Q4RDNA_CFG_OVERLAP_PREVIOUS;
        return v;
    }();
    return &c;
}
}  // namespace

extern "C" {

int q4rdna_mul_mat(const char *weight_name, int64_t weight_ne0, int64_t weight_ne1, const float *x, int64_t x_ne0,
                   float *y, int64_t y_ne0, q4rdna_stream_t stream) {
    if (x == nullptr || y == nullptr) return 0;
    Registry &r = registry();
    std::lock_guard<std::mutex> lock(r.mu);
    Found f;
    if (!find(r, weight_name, weight_ne0, weight_ne1, (cudaStream_t)stream, f)) return 0;
    if (x_ne0 != (int64_t)f.entry->cols || y_ne0 != (int64_t)f.entry->rows) {
        std::fprintf(stderr, "Q4_RDNA: shape mismatch for %s\n", weight_name);
        return 0;
    }
    void *ws = stream_workspace(r, (cudaStream_t)stream);
    if (r.ws_bytes && ws == nullptr) return 0;
    if (q4rdna_gemv(f.tiles, x, y, (int)f.entry->rows, (int)f.entry->cols, 1, hook_cfg(), ws, r.ws_bytes, stream) !=
        Q4RDNA_OK)
        return 0;
    g_op_launches.fetch_add(1, std::memory_order_relaxed);
    f.entry->hits->fetch_add(1, std::memory_order_relaxed);
    return 1;
}

int q4rdna_mul_mat_add(const char *weight_name, int64_t weight_ne0, int64_t weight_ne1, const float *x,
                       int64_t x_ne0, const float *add, int64_t add_nelements, float *y, int64_t y_nelements,
                       q4rdna_stream_t stream) {
    if (x == nullptr || y == nullptr || add == nullptr) return 0;
    Registry &r = registry();
    std::lock_guard<std::mutex> lock(r.mu);
    Found f;
    if (!find(r, weight_name, weight_ne0, weight_ne1, (cudaStream_t)stream, f)) return 0;
    if (x_ne0 != (int64_t)f.entry->cols || add_nelements != (int64_t)f.entry->rows ||
        y_nelements != (int64_t)f.entry->rows)
        return 0;
    void *ws = stream_workspace(r, (cudaStream_t)stream);
    if (r.ws_bytes && ws == nullptr) return 0;
    if (q4rdna_gemv_add(f.tiles, x, add, y, (int)f.entry->rows, (int)f.entry->cols, 1, hook_cfg(), ws, r.ws_bytes,
                        stream) != Q4RDNA_OK)
        return 0;
    g_op_launches.fetch_add(1, std::memory_order_relaxed);
    f.entry->hits->fetch_add(1, std::memory_order_relaxed);
    return 1;
}

int q4rdna_mul_mat_glu(const char *up_name, int64_t up_ne0, int64_t up_ne1, const char *gate_name, int64_t gate_ne0,
                       int64_t gate_ne1, const float *x, int64_t x_ne0, float *y, int64_t y_nelements,
                       q4rdna_stream_t stream) {
    if (x == nullptr || y == nullptr) return 0;
    Registry &r = registry();
    std::lock_guard<std::mutex> lock(r.mu);
    Found up, gate;
    if (!find(r, up_name, up_ne0, up_ne1, (cudaStream_t)stream, up) || !find(r, gate_name, gate_ne0, gate_ne1, (cudaStream_t)stream, gate)) return 0;
    if (up.entry->rows != gate.entry->rows || up.entry->cols != gate.entry->cols ||
        x_ne0 != (int64_t)up.entry->cols || y_nelements != (int64_t)up.entry->rows)
        return 0;
    void *ws = stream_workspace(r, (cudaStream_t)stream);
    if (r.ws_bytes && ws == nullptr) return 0;
    if (q4rdna_gemv_swiglu(up.tiles, gate.tiles, x, y, (int)up.entry->rows, (int)up.entry->cols, 1, hook_cfg(), ws,
                           r.ws_bytes, stream) != Q4RDNA_OK)
        return 0;
    g_op_launches.fetch_add(1, std::memory_order_relaxed);
    up.entry->hits->fetch_add(1, std::memory_order_relaxed);
    gate.entry->hits->fetch_add(1, std::memory_order_relaxed);
    return 1;
}

uint64_t q4rdna_registry_hits(const char *weight_name) {
    Registry &r = registry();
    std::lock_guard<std::mutex> lock(r.mu);
    if (r.sc == nullptr || weight_name == nullptr) return 0;
    const auto it = r.sc->index.find(weight_name);
    return it == r.sc->index.end() ? 0 : r.sc->entries[it->second].hits->load();
}

// Exit-time summary in the reference's format (source/q4rdna.cu:75-112).
void q4rdna_report_stats(void) {
    const uint64_t launches = g_op_launches.load();
    if (launches != 0)
        std::fprintf(stderr, "Q4_RDNA: launched %llu decode GEMV kernels\n", (unsigned long long)launches);
    Registry &r = registry();
    std::lock_guard<std::mutex> lock(r.mu);
    if (r.sc == nullptr) return;
    uint64_t s12288_4096 = 0, s4096_12288 = 0, s4096_4096 = 0, s1024_4096 = 0, other = 0;
    unsigned unique = 0;
    const bool trace = std::getenv("LLAMA_Q4_RDNA_TRACE") != nullptr;
    for (const Entry &e : r.sc->entries) {
        const uint64_t hits = e.hits->load();
        if (hits == 0) continue;
        ++unique;
        if (e.rows == 12288 && e.cols == 4096) s12288_4096 += hits;
        else if (e.rows == 4096 && e.cols == 12288) s4096_12288 += hits;
        else if (e.rows == 4096 && e.cols == 4096) s4096_4096 += hits;
        else if (e.rows == 1024 && e.cols == 4096) s1024_4096 += hits;
        else other += hits;
        if (trace) std::fprintf(stderr, "Q4_RDNA: hit %-31s %llu\n", e.name.c_str(), (unsigned long long)hits);
    }
    std::fprintf(stderr,
                 "Q4_RDNA: unique=%u, hits by rows x columns: 12288x4096=%llu, 4096x12288=%llu, "
                 "4096x4096=%llu, 1024x4096=%llu, other=%llu\n",
                 unique, (unsigned long long)s12288_4096, (unsigned long long)s4096_12288,
                 (unsigned long long)s4096_4096, (unsigned long long)s1024_4096, (unsigned long long)other);
}

void q4rdna_registry_reset(void) {
    noalloc_forget_devices();
    Registry &r = registry();
    std::lock_guard<std::mutex> lock(r.mu);
    for (auto &kv : r.ws) cudaFree(kv.second);
    r.ws.clear();
    if (r.sc) q4rdna_sidecar_close(r.sc);
    r.sc = nullptr;
    r.ws_bytes = 0;
    r.attempted = false;
    g_op_launches.store(0);
}

}  // extern "C"
