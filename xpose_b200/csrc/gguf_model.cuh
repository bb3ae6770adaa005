// Real weights: a GGUF model file read in place (mmap), its tensors
// dequantised on the device from their ggml block types and packed to the
// KM4 + bf16 planes the engine streams, and the reference's packed-weight
// cache ("<model>.xpack") read and written in its own on-disk format, so a
// cache either side writes is valid for the other.
//
// Mirrors the reference load path examples/llm/decode.cpp:1418-1535 (config
// from the file's metadata, norm weights stored as (1 + w) and loaded back as
// w, the 26 x 7 + 1 pack tasks in decode.cpp:985-1036 order, tied output
// head) and the cache of decode.cpp:711-1328 (header, entry table, per-entry
// hash, source stamp, ".tmp" + rename). Packing runs on the GPU (the device
// packer is bit-exact with the reference's host packer), not on host threads.
#pragma once
#include <cuda_fp16.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstring>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "engine.cuh"
#include "quant.cuh"

namespace xp {

// ---- GGUF reader (the published v2/v3 layout) ----------------------------------
struct GgufTensor {
    std::string name;
    std::vector<uint64_t> shape;  // fastest dimension first
    uint32_t type = 0;
    uint64_t offset = 0;          // from the start of the data section
    const uint8_t* data = nullptr;
    uint64_t nbytes = 0;
    uint64_t elements() const {
        uint64_t n = 1;
        for (uint64_t d : shape) n *= d;
        return n;
    }
};
struct GgufValue {
    uint32_t type = 0;   // gguf metadata type
    uint64_t u = 0;      // integers and bools
    double f = 0;        // floats
    std::string s;       // strings
    uint64_t count = 0;  // arrays: element count
    uint32_t elem_type = 0;         // arrays: element type
    std::vector<std::string> strs;  // string arrays
    std::vector<double> nums;       // numeric arrays
};

class GgufFile {
   public:
    std::string path;
    std::unordered_map<std::string, GgufValue> kv;
    std::vector<GgufTensor> tensors;
    const uint8_t* base = nullptr;
    size_t size = 0;

    ~GgufFile() {
        if (base) munmap(const_cast<uint8_t*>(base), size);
    }
    const GgufTensor* tensor(const std::string& n) const {
        for (const auto& t : tensors)
            if (t.name == n) return &t;
        return nullptr;
    }
    bool get_u(const std::string& k, uint64_t& v) const {
        auto it = kv.find(k);
        if (it == kv.end() || it->second.type == 8 || it->second.type == 9) return false;
        v = (it->second.type == 6 || it->second.type == 12) ? (uint64_t)it->second.f : it->second.u;
        return true;
    }
    bool get_f(const std::string& k, double& v) const {
        auto it = kv.find(k);
        if (it == kv.end() || it->second.type == 8 || it->second.type == 9) return false;
        v = (it->second.type == 6 || it->second.type == 12) ? it->second.f : (double)it->second.u;
        return true;
    }
    std::string get_s(const std::string& k) const {
        auto it = kv.find(k);
        return it == kv.end() || it->second.type != 8 ? std::string() : it->second.s;
    }

    xp_status open(const char* p) {
        path = p;
        const int fd = ::open(p, O_RDONLY);
        if (fd < 0) return fail(XP_ERR_INVALID, "gguf: cannot open '%s': %s", p, std::strerror(errno));
        struct stat st {};
        if (fstat(fd, &st) != 0 || st.st_size < 24) {
            ::close(fd);
            return fail(XP_ERR_INVALID, "gguf: '%s' is too short", p);
        }
        size = (size_t)st.st_size;
        void* m = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (m == MAP_FAILED) return fail(XP_ERR_INVALID, "gguf: cannot map '%s'", p);
        base = static_cast<const uint8_t*>(m);
        return parse();
    }

   private:
    size_t pos = 0;
    bool need(size_t n) const { return pos + n <= size; }
    template <class T> bool rd(T& v) {
        if (!need(sizeof(T))) return false;
        std::memcpy(&v, base + pos, sizeof(T));
        pos += sizeof(T);
        return true;
    }
    bool rd_str(std::string& s, uint32_t version) {
        uint64_t n = 0;
        if (version == 1) {
            uint32_t n32;
            if (!rd(n32)) return false;
            n = n32;
        } else if (!rd(n)) {
            return false;
        }
        if (!need(n)) return false;
        s.assign(reinterpret_cast<const char*>(base + pos), n);
        pos += n;
        return true;
    }
    static size_t scalar_size(uint32_t t) {
        switch (t) {
            case 0: case 1: case 7: return 1;
            case 2: case 3: return 2;
            case 4: case 5: case 6: return 4;
            case 10: case 11: case 12: return 8;
            default: return 0;
        }
    }
    bool rd_scalar(uint32_t t, GgufValue& v) {
        const size_t sz = scalar_size(t);
        if (!sz || !need(sz)) return false;
        uint64_t raw = 0;
        std::memcpy(&raw, base + pos, sz);
        pos += sz;
        if (t == 6) { float f; std::memcpy(&f, &raw, 4); v.f = f; }
        else if (t == 12) { double d; std::memcpy(&d, &raw, 8); v.f = d; }
        else if (t == 1) v.u = (uint64_t)(int64_t)(int8_t)raw;
        else if (t == 3) v.u = (uint64_t)(int64_t)(int16_t)raw;
        else if (t == 5) v.u = (uint64_t)(int64_t)(int32_t)raw;
        else v.u = raw;
        return true;
    }
    xp_status bad(const char* what) { return fail(XP_ERR_INVALID, "gguf: '%s': %s", path.c_str(), what); }

    xp_status parse() {
        uint32_t magic = 0, version = 0;
        if (!rd(magic) || magic != 0x46554747u) return bad("not a GGUF file (bad magic)");
        if (!rd(version) || version < 2 || version > 3) return bad("unsupported GGUF version (2 or 3 expected)");
        uint64_t nt = 0, nkv = 0;
        if (!rd(nt) || !rd(nkv) || nt > (1u << 20) || nkv > (1u << 20)) return bad("implausible header counts");
        for (uint64_t i = 0; i < nkv; ++i) {
            std::string key;
            uint32_t t = 0;
            if (!rd_str(key, version) || !rd(t)) return bad("truncated metadata");
            GgufValue v;
            v.type = t;
            if (t == 8) {
                if (!rd_str(v.s, version)) return bad("truncated string value");
            } else if (t == 9) {
                uint32_t et = 0;
                uint64_t n = 0;
                if (!rd(et) || !rd(n)) return bad("truncated array");
                v.count = n;
                v.elem_type = et;
                if (et == 8) {
                    if (n > size) return bad("implausible string array");
                    v.strs.resize(n);
                    for (uint64_t k = 0; k < n; ++k)
                        if (!rd_str(v.strs[k], version)) return bad("truncated string array");
                } else {
                    const size_t sz = scalar_size(et);
                    if (!sz || n > size || !need(sz * n)) return bad("truncated or nested array");
                    v.nums.resize(n);
                    for (uint64_t k = 0; k < n; ++k) {
                        GgufValue e;
                        rd_scalar(et, e);
                        v.nums[k] = (et == 6 || et == 12) ? e.f : (et == 1 || et == 3 || et == 5 || et == 11)
                                                                      ? (double)(int64_t)e.u : (double)e.u;
                    }
                }
            } else if (!rd_scalar(t, v)) {
                return bad("bad metadata value");
            }
            kv[key] = std::move(v);
        }
        for (uint64_t i = 0; i < nt; ++i) {
            GgufTensor t;
            uint32_t nd = 0;
            if (!rd_str(t.name, version) || !rd(nd) || nd == 0 || nd > 4) return bad("bad tensor info");
            t.shape.resize(nd);
            for (auto& d : t.shape)
                if (!rd(d)) return bad("truncated tensor shape");
            if (!rd(t.type) || !rd(t.offset)) return bad("truncated tensor info");
            tensors.push_back(std::move(t));
        }
        uint64_t align = 32;
        get_u("general.alignment", align);
        if (align == 0 || (align & (align - 1))) return bad("general.alignment is not a power of two");
        const size_t data0 = (pos + align - 1) / align * align;
        for (auto& t : tensors) {
            const GgmlType* g = ggml_type(t.type);
            if (!g) continue;  // a type the loader does not read; fails only if a needed tensor has it
            const uint64_t n = t.elements();
            if (n % g->block) return bad("a tensor's size is not a whole number of blocks");
            t.nbytes = n / g->block * g->bytes;
            if (data0 + t.offset + t.nbytes > size) return bad("a tensor runs past the end of the file");
            t.data = base + data0 + t.offset;
        }
        return XP_OK;
    }
};

// ---- the .xpack cache (decode.cpp:711-1328) ------------------------------------
// The on-disk layout is the reference's, field for field, so either side's
// cache is accepted by the other: a 128-byte header, the entries' payloads
// (nibble words then scale words, contiguous, in pack-task order), then the
// entry table; a per-entry FNV-1a-style hash over 4 MiB chunks.
struct XpackHeader {
    char magic[8];
    uint32_t version, header_size;
    uint64_t src_size, src_mtime_ns, src_fingerprint;
    uint32_t layout, qblock, group, scale_bf16, packer_version, n_entries;
    uint64_t table_offset, total_size;
    uint64_t reserved[6];
};
static_assert(sizeof(XpackHeader) == 128, "the .xpack header is 128 bytes");
struct XpackEntry {
    char name[80];
    uint32_t rows, cols;
    uint64_t offset, words_bytes, scale_bytes, hash;
};
static_assert(sizeof(XpackEntry) == 120, "an .xpack entry is 120 bytes");
constexpr char kXpackMagic[8] = {'X', 'P', 'A', 'C', 'K', '0', '0', '1'};
constexpr uint32_t kXpackLayoutKm4Bf16 = 2;   // MatvecLayout::Km4Bf16
constexpr uint64_t kXpackChunk = 4ull << 20;  // hash chunk (part of the format)
constexpr uint64_t kFnvPrime = 1099511628211ull, kFnvBasis = 1469598103934665603ull;

inline uint64_t xpack_hash64(const uint8_t* p, uint64_t n) {
    uint64_t h = kFnvBasis ^ n, i = 0;
    for (; i + 8 <= n; i += 8) {
        uint64_t w;
        std::memcpy(&w, p + i, 8);
        h = (h ^ w) * kFnvPrime;
        h ^= h >> 29;
    }
    for (; i < n; ++i) h = (h ^ p[i]) * kFnvPrime;
    h ^= h >> 32;
    h *= 0xff51afd7ed558ccdull;
    h ^= h >> 32;
    return h;
}
// chunk hashes computed on host threads, folded in chunk order
inline uint64_t xpack_hash_chunks(const void* data, uint64_t n) {
    const uint8_t* p = static_cast<const uint8_t*>(data);
    const uint64_t nc = (n + kXpackChunk - 1) / kXpackChunk;
    std::vector<uint64_t> part(nc);
    const unsigned nt = (unsigned)std::min<uint64_t>(std::max(1u, std::thread::hardware_concurrency()), nc);
    std::atomic<uint64_t> next{0};
    auto work = [&]() {
        for (uint64_t c; (c = next.fetch_add(1)) < nc;)
            part[c] = xpack_hash64(p + c * kXpackChunk, std::min(kXpackChunk, n - c * kXpackChunk));
    };
    std::vector<std::thread> pool;
    for (unsigned i = 1; i < nt; ++i) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
    uint64_t acc = kFnvBasis ^ n;
    for (uint64_t v : part) acc = (acc ^ v) * kFnvPrime;
    return acc;
}
// size, mtime and a hash of the first and last 64 KiB of the source model
inline bool xpack_source_stamp(const std::string& path, XpackHeader& h) {
    struct stat st {};
    if (::stat(path.c_str(), &st) != 0) return false;
    h.src_size = (uint64_t)st.st_size;
    h.src_mtime_ns = (uint64_t)st.st_mtim.tv_sec * 1000000000ull + (uint64_t)st.st_mtim.tv_nsec;
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) return false;
    std::vector<uint8_t> buf(std::min<uint64_t>(64 << 10, h.src_size));
    uint64_t f = h.src_size;
    for (int which = 0; which < 2; ++which) {
        const off_t off = which == 0 ? 0 : (off_t)(h.src_size - buf.size());
        if (pread(fd, buf.data(), buf.size(), off) != (ssize_t)buf.size()) {
            ::close(fd);
            return false;
        }
        f = xpack_hash64(buf.data(), buf.size()) ^ (f * kFnvPrime);
    }
    ::close(fd);
    h.src_fingerprint = f;
    return true;
}

struct PackTask {
    std::string name;
    uint32_t rows, cols;
    const GgufTensor* t;
};
struct PackedPlanes {
    std::vector<uint32_t> words, scales;
};

// The cache's payload for `tasks` if the file at `cpath` is valid for them and
// this model, else an empty vector and the reason.
inline bool xpack_read(const std::string& cpath, const XpackHeader& want, const std::vector<PackTask>& tasks,
                       std::vector<PackedPlanes>& out, std::string& why) {
    const int fd = ::open(cpath.c_str(), O_RDONLY);
    if (fd < 0) { why = "no cache file"; return false; }
    auto reject = [&](const char* w) { why = w; ::close(fd); return false; };
    struct stat st {};
    if (fstat(fd, &st) != 0) return reject("stat failed");
    XpackHeader h{};
    if (pread(fd, &h, sizeof h, 0) != (ssize_t)sizeof h) return reject("truncated header");
    if (std::memcmp(h.magic, kXpackMagic, 8)) return reject("bad magic");
    if (h.version != 1 || h.header_size != sizeof(XpackHeader)) return reject("version or header size mismatch");
    if (h.src_size != want.src_size || h.src_mtime_ns != want.src_mtime_ns) return reject("model size or mtime changed");
    if (h.src_fingerprint != want.src_fingerprint) return reject("model contents changed");
    if (h.layout != want.layout || h.qblock != want.qblock || h.group != want.group ||
        h.scale_bf16 != want.scale_bf16 || h.packer_version != want.packer_version)
        return reject("packing layout or packer version differs");
    if (h.n_entries != tasks.size() || h.n_entries == 0 || h.n_entries > 8192) return reject("tensor count differs");
    if (h.total_size != (uint64_t)st.st_size) return reject("file size mismatch");
    if (h.table_offset < sizeof(XpackHeader) ||
        h.table_offset + (uint64_t)h.n_entries * sizeof(XpackEntry) != h.total_size)
        return reject("table does not close the file");
    std::vector<XpackEntry> table(h.n_entries);
    const size_t tb = table.size() * sizeof(XpackEntry);
    if (pread(fd, table.data(), tb, (off_t)h.table_offset) != (ssize_t)tb) return reject("truncated table");
    uint64_t off = sizeof(XpackHeader);
    for (size_t i = 0; i < tasks.size(); ++i) {
        const XpackEntry& e = table[i];
        if (tasks[i].name.size() >= sizeof e.name || std::memcmp(e.name, tasks[i].name.c_str(), tasks[i].name.size() + 1))
            return reject("tensor name/order mismatch");
        if (e.rows != tasks[i].rows || e.cols != tasks[i].cols) return reject("tensor shape mismatch");
        const uint64_t wb = (uint64_t)e.rows * e.cols / 2, sb = (uint64_t)e.rows / 128 * e.cols * 8;
        if (e.words_bytes != wb || e.scale_bytes != sb) return reject("entry byte count disagrees with its shape");
        if (e.offset != off) return reject("entry offsets not contiguous");
        off += wb + sb;
    }
    if (off != h.table_offset) return reject("payload does not reach the table");
    out.resize(tasks.size());
    for (size_t i = 0; i < tasks.size(); ++i) {
        const XpackEntry& e = table[i];
        PackedPlanes& pp = out[i];
        pp.words.resize(e.words_bytes / 4);
        pp.scales.resize(e.scale_bytes / 4);
        if (pread(fd, pp.words.data(), e.words_bytes, (off_t)e.offset) != (ssize_t)e.words_bytes ||
            pread(fd, pp.scales.data(), e.scale_bytes, (off_t)(e.offset + e.words_bytes)) != (ssize_t)e.scale_bytes) {
            out.clear();
            return reject("truncated payload");
        }
        const uint64_t hh = xpack_hash_chunks(pp.words.data(), e.words_bytes) ^
                            (xpack_hash_chunks(pp.scales.data(), e.scale_bytes) * kFnvPrime);
        if (hh != e.hash) {
            out.clear();
            return reject("an entry failed its checksum");
        }
    }
    ::close(fd);
    return true;
}

// Writes `<cpath>.tmp` then renames it into place (a partial file is never
// visible under the cache's name).
inline bool xpack_write(const std::string& cpath, XpackHeader h, const std::vector<PackTask>& tasks,
                        const std::vector<PackedPlanes>& planes, std::string& why) {
    const std::string tmp = cpath + ".tmp";
    const int fd = ::open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) { why = std::string("cannot write ") + tmp + ": " + std::strerror(errno); return false; }
    auto put = [&](const void* p, size_t n) {
        const uint8_t* b = static_cast<const uint8_t*>(p);
        for (size_t done = 0; done < n;) {
            const ssize_t r = ::write(fd, b + done, n - done);
            if (r <= 0) return false;
            done += (size_t)r;
        }
        return true;
    };
    XpackHeader blank{};
    bool ok = put(&blank, sizeof blank);
    std::vector<XpackEntry> table(tasks.size());
    uint64_t off = sizeof(XpackHeader);
    for (size_t i = 0; ok && i < tasks.size(); ++i) {
        XpackEntry& e = table[i];
        std::memset(&e, 0, sizeof e);
        std::snprintf(e.name, sizeof e.name, "%s", tasks[i].name.c_str());
        e.rows = tasks[i].rows;
        e.cols = tasks[i].cols;
        e.offset = off;
        e.words_bytes = planes[i].words.size() * 4;
        e.scale_bytes = planes[i].scales.size() * 4;
        e.hash = xpack_hash_chunks(planes[i].words.data(), e.words_bytes) ^
                 (xpack_hash_chunks(planes[i].scales.data(), e.scale_bytes) * kFnvPrime);
        ok = put(planes[i].words.data(), e.words_bytes) && put(planes[i].scales.data(), e.scale_bytes);
        off += e.words_bytes + e.scale_bytes;
    }
    h.table_offset = off;
    h.total_size = off + table.size() * sizeof(XpackEntry);
    ok = ok && put(table.data(), table.size() * sizeof(XpackEntry)) && lseek(fd, 0, SEEK_SET) == 0 &&
         put(&h, sizeof h) && fsync(fd) == 0;
    ::close(fd);
    if (!ok || ::rename(tmp.c_str(), cpath.c_str()) != 0) {
        why = std::string("could not finish the cache: ") + std::strerror(errno);
        ::unlink(tmp.c_str());
        return false;
    }
    return true;
}

}  // namespace xp

// ---- C ABI ---------------------------------------------------------------------
extern "C" {

xp_status xp_gguf_dequantize(void* stream, uint32_t type_id, const void* src, float* dst, uint64_t n) {
    using namespace xp;
    if (!src || !dst) return fail(XP_ERR_INVALID, "xp_gguf_dequantize: null pointer");
    const GgmlType* g = xp::ggml_type(type_id);
    if (!g) return fail(XP_ERR_UNSUPPORTED, "xp_gguf_dequantize: ggml type %u is not dequantised", type_id);
    if (n % g->block) return fail(XP_ERR_INVALID, "xp_gguf_dequantize: %llu is not a whole number of %s blocks",
                                  (unsigned long long)n, g->name);
    if (n == 0) return XP_OK;
    return cuda_status(gguf_dequant((cudaStream_t)stream, type_id, src, dst, n), "gguf_dequantize");
}

xp_status xp_quant_repack_sizes(uint32_t type_id, uint32_t rows, uint32_t cols, uint64_t* sizes) {
    using namespace xp;
    if (!sizes) return fail(XP_ERR_INVALID, "xp_quant_repack_sizes: null sizes");
    if (!quant::repack_sizes(type_id, rows, cols, sizes))
        return fail(XP_ERR_INVALID, "xp_quant_repack: type %u with %u x %u is not repackable (Q8_0, Q5_0: cols %% 32; "
                    "Q4_K, Q6_K: cols %% 256)", type_id, rows, cols);
    return XP_OK;
}

xp_status xp_quant_repack(void* stream, uint32_t type_id, const void* src, uint32_t rows, uint32_t cols, uint32_t* q,
                          uint32_t* high, float* scale, float* bias) {
    using namespace xp;
    uint64_t sizes[4];
    if (xp_status e = xp_quant_repack_sizes(type_id, rows, cols, sizes); e != XP_OK) return e;
    if (!src || !q || !scale || (sizes[1] && !high) || (sizes[3] && !bias))
        return fail(XP_ERR_INVALID, "xp_quant_repack: null pointer for a plane this type has");
    if (((uintptr_t)q) & 15) return fail(XP_ERR_INVALID, "xp_quant_repack: the quant plane must be 16-byte aligned");
    quant::RepackArgs a{};
    a.src = static_cast<const uint8_t*>(src);
    a.quant = reinterpret_cast<uint4*>(q);
    a.high = high;
    a.scale = scale;
    a.bias = bias;
    a.type = type_id;
    a.rows = rows;
    a.cols = cols;
    a.nkb = cols / 32;
    a.slots = (uint32_t)(sizes[2] / (type_id == 14 ? 2 : 1));
    quant::repack_kernel<<<(a.slots + 255) / 256, 256, 0, (cudaStream_t)stream>>>(a);
    return cuda_status(cudaGetLastError(), "quant_repack");
}

xp_status xp_session_create_gguf(int device, const char* gguf_path, const xp_model_config* policy,
                                 const xp_sampling* sp, const char* pack_cache, xp_session** out) {
    using namespace xp;
    if (!gguf_path || !sp || !out) return fail(XP_ERR_INVALID, "xp_session_create_gguf: null argument");
    *out = nullptr;
    XP_CUDA_TRY(cudaSetDevice(device));
    GgufFile f;
    if (xp_status s = f.open(gguf_path); s != XP_OK) return s;

    // shapes from the file (DecodeConfig::from_model, decode.cpp:258-275),
    // policy fields from the caller, Gemma-3-1B defaults otherwise
    xp_model_config c{26, 1152, 6912, 4, 1, 256, 262144, 8192, 512, 6, 1e-6f, 1e6f, 1e4f, 0.0f, 0.0f};
    const std::string arch = f.get_s("general.architecture").empty() ? "gemma3" : f.get_s("general.architecture");
    auto U = [&](const char* k, uint32_t& dst) {
        uint64_t v;
        if (f.get_u(arch + "." + k, v) && v) dst = (uint32_t)v;
    };
    U("block_count", c.n_layers);
    U("attention.head_count", c.n_heads);
    U("attention.head_count_kv", c.n_kv_heads);
    U("embedding_length", c.hidden);
    U("feed_forward_length", c.ffn);
    U("attention.key_length", c.head_dim);
    U("attention.sliding_window", c.sliding_window);
    double fv;
    if (f.get_f(arch + ".attention.layer_norm_rms_epsilon", fv)) c.rms_eps = (float)fv;
    if (f.get_f(arch + ".rope.freq_base", fv)) c.rope_theta_global = (float)fv;
    auto tok = f.kv.find("tokenizer.ggml.tokens");
    if (tok != f.kv.end() && tok->second.type == 9 && tok->second.count) c.vocab = (uint32_t)tok->second.count;
    if (policy) {
        if (policy->max_seq) c.max_seq = policy->max_seq;
        c.global_every = policy->global_every;
        if (policy->sliding_window) c.sliding_window = policy->sliding_window;
        if (policy->rope_theta_local > 0) c.rope_theta_local = policy->rope_theta_local;
        c.embed_scale = policy->embed_scale;
        c.attn_scale = policy->attn_scale;
    }
    const uint32_t H = c.hidden, QD = c.n_heads * c.head_dim, KVD = c.n_kv_heads * c.head_dim, F = c.ffn;

    // the pack tasks, in the reference's order (decode.cpp:1023-1036)
    std::vector<PackTask> tasks;
    auto add = [&](const std::string& name, uint32_t rows, uint32_t cols) -> xp_status {
        const GgufTensor* t = f.tensor(name);
        if (!t) return fail(XP_ERR_INVALID, "gguf: missing tensor '%s'", name.c_str());
        if (t->shape.size() != 2 || t->shape[0] != rows || t->shape[1] != cols)
            return fail(XP_ERR_INVALID, "gguf: tensor '%s' has an unexpected shape (want {%u,%u})", name.c_str(), rows,
                        cols);
        if (!t->data) return fail(XP_ERR_UNSUPPORTED, "gguf: tensor '%s' has ggml type %u, which is not read",
                                  name.c_str(), t->type);
        if (rows % 128 || cols % 64)
            return fail(XP_ERR_INVALID, "gguf: tensor '%s' is %u x %u; the packing needs rows %% 128 and cols %% 64 == 0",
                        name.c_str(), rows, cols);
        tasks.push_back({name, rows, cols, t});
        return XP_OK;
    };
    const char* mats[7] = {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"};
    const uint32_t shp[7][2] = {{H, QD}, {H, KVD}, {H, KVD}, {QD, H}, {H, F}, {H, F}, {F, H}};
    for (uint32_t l = 0; l < c.n_layers; ++l)
        for (int m = 0; m < 7; ++m)
            if (xp_status s = add("blk." + std::to_string(l) + "." + mats[m] + ".weight", shp[m][0], shp[m][1]); s != XP_OK)
                return s;
    const bool untied = f.tensor("output.weight") != nullptr;
    if (xp_status s = add(untied ? "output.weight" : "token_embd.weight", H, c.vocab); s != XP_OK) return s;
    const GgufTensor* emb = f.tensor("token_embd.weight");
    if (!emb || !emb->data || emb->elements() != (uint64_t)H * c.vocab)
        return fail(XP_ERR_INVALID, "gguf: token_embd.weight is missing, of an unread type, or not hidden x vocab");

    cudaStream_t st = nullptr;
    XP_CUDA_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    std::vector<void*> dev;
    auto dalloc = [&](size_t n) -> void* {
        void* p = nullptr;
        if (cudaMalloc(&p, n) != cudaSuccess) return nullptr;
        dev.push_back(p);
        return p;
    };
    auto cleanup = [&]() {
        cudaStreamSynchronize(st);
        for (void* p : dev) cudaFree(p);
        cudaStreamDestroy(st);
    };
    // whole tensor -> fp32 host vector through the device dequantiser
    auto dequant_host = [&](const GgufTensor& t, std::vector<float>& h, float* dfp = nullptr) -> xp_status {
        void* draw = dalloc(t.nbytes);
        float* dst = dfp ? dfp : static_cast<float*>(dalloc(t.elements() * 4));
        if (!draw || !dst) return fail(XP_ERR_OOM, "gguf: device buffers for '%s'", t.name.c_str());
        XP_CUDA_TRY(cudaMemcpyAsync(draw, t.data, t.nbytes, cudaMemcpyHostToDevice, st));
        XP_CUDA_TRY(gguf_dequant(st, t.type, draw, dst, t.elements()));
        h.resize(t.elements());
        XP_CUDA_TRY(cudaMemcpyAsync(h.data(), dst, t.elements() * 4, cudaMemcpyDeviceToHost, st));
        XP_CUDA_TRY(cudaStreamSynchronize(st));
        cudaFree(draw);
        dev.erase(std::find(dev.begin(), dev.end(), draw));
        if (!dfp) {
            cudaFree(dst);
            dev.erase(std::find(dev.begin(), dev.end(), static_cast<void*>(dst)));
        }
        return XP_OK;
    };

    // norms: stored as (1 + w), loaded back as w (decode.cpp:1480-1502)
    std::vector<std::vector<float>> norms;
    auto load_norm = [&](const std::string& name, uint32_t n) -> xp_status {
        const GgufTensor* t = f.tensor(name);
        if (!t || !t->data || t->elements() != n)
            return fail(XP_ERR_INVALID, "gguf: norm tensor '%s' missing, of an unread type, or not %u elements",
                        name.c_str(), n);
        std::vector<float> h;
        if (xp_status s = dequant_host(*t, h); s != XP_OK) return s;
        for (float& v : h) v -= 1.0f;
        norms.push_back(std::move(h));
        return XP_OK;
    };
    const char* nn[6] = {"attn_norm", "post_attention_norm", "ffn_norm", "post_ffw_norm", "attn_q_norm", "attn_k_norm"};
    xp_status s = XP_OK;
    for (uint32_t l = 0; l < c.n_layers && s == XP_OK; ++l)
        for (int k = 0; k < 6 && s == XP_OK; ++k)
            s = load_norm("blk." + std::to_string(l) + "." + nn[k] + ".weight", k < 4 ? H : c.head_dim);
    if (s == XP_OK) s = load_norm("output_norm.weight", H);
    std::vector<float> embed;
    if (s == XP_OK) s = dequant_host(*emb, embed);
    if (s != XP_OK) { cleanup(); return s; }

    // packed planes: from a valid cache, else packed on the device (and cached)
    XpackHeader want{};
    std::memcpy(want.magic, kXpackMagic, 8);
    want.version = 1;
    want.header_size = sizeof(XpackHeader);
    want.layout = kXpackLayoutKm4Bf16;
    want.qblock = 32;
    want.group = 64;
    want.scale_bf16 = 1;
    want.packer_version = 1;
    want.n_entries = (uint32_t)tasks.size();
    const std::string cpath = pack_cache ? std::string(pack_cache) : std::string(gguf_path) + ".xpack";
    const bool use_cache = !cpath.empty() && xpack_source_stamp(gguf_path, want);
    std::vector<PackedPlanes> planes;
    std::string info;
    bool from_cache = false, written = false;
    if (use_cache) {
        std::string why;
        from_cache = xpack_read(cpath, want, tasks, planes, why);
        info = from_cache ? "loaded packed weights from " + cpath : "repacked (cache: " + why + ")";
    } else {
        info = "repacked (no cache)";
    }
    if (!from_cache) {
        planes.assign(tasks.size(), PackedPlanes{});
        for (size_t i = 0; i < tasks.size() && s == XP_OK; ++i) {
            const PackTask& t = tasks[i];
            void* draw = dalloc(t.t->nbytes);
            float* dw = static_cast<float*>(dalloc((size_t)t.rows * t.cols * 4));
            uint32_t* dwq = static_cast<uint32_t*>(dalloc((size_t)t.rows * t.cols / 2));
            uint32_t* dsc = static_cast<uint32_t*>(dalloc((size_t)t.rows / 128 * t.cols * 8));
            if (!draw || !dw || !dwq || !dsc) { s = fail(XP_ERR_OOM, "gguf: device buffers for packing"); break; }
            cudaError_t e = cudaMemcpyAsync(draw, t.t->data, t.t->nbytes, cudaMemcpyHostToDevice, st);
            if (e == cudaSuccess) e = gguf_dequant(st, t.t->type, draw, dw, t.t->elements());
            if (e != cudaSuccess) { s = cuda_status(e, "gguf: dequantise"); break; }
            if ((s = xp_pack_km4bf16(st, dw, t.rows, t.cols, dwq, dsc)) != XP_OK) break;
            planes[i].words.resize((size_t)t.rows * t.cols / 8);
            planes[i].scales.resize((size_t)t.rows / 128 * t.cols * 2);
            e = cudaMemcpyAsync(planes[i].words.data(), dwq, planes[i].words.size() * 4, cudaMemcpyDeviceToHost, st);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(planes[i].scales.data(), dsc, planes[i].scales.size() * 4, cudaMemcpyDeviceToHost, st);
            if (e == cudaSuccess) e = cudaStreamSynchronize(st);
            if (e != cudaSuccess) { s = cuda_status(e, "gguf: pack"); break; }
            for (void* p : {draw, static_cast<void*>(dw), static_cast<void*>(dwq), static_cast<void*>(dsc)}) {
                cudaFree(p);
                dev.erase(std::find(dev.begin(), dev.end(), p));
            }
        }
        if (s == XP_OK && use_cache) {
            std::string why;
            written = xpack_write(cpath, want, tasks, planes, why);
            info += written ? "; wrote " + cpath : "; " + why;
        }
    }
    cleanup();
    if (s != XP_OK) return s;

    std::vector<xp_layer_weights> L(c.n_layers);
    for (uint32_t l = 0; l < c.n_layers; ++l) {
        for (int m = 0; m < 7; ++m) {
            L[l].words[m] = planes[l * 7 + m].words.data();
            L[l].scales[m] = planes[l * 7 + m].scales.data();
        }
        L[l].attn_norm = norms[l * 6 + 0].data();
        L[l].post_attn_norm = norms[l * 6 + 1].data();
        L[l].ffn_norm = norms[l * 6 + 2].data();
        L[l].post_ffn_norm = norms[l * 6 + 3].data();
        L[l].q_norm = norms[l * 6 + 4].data();
        L[l].k_norm = norms[l * 6 + 5].data();
    }
    const PackedPlanes& lm = planes.back();
    if ((s = xp_session_create(device, &c, sp, L.data(), lm.words.data(), lm.scales.data(), norms.back().data(),
                               embed.data(), out)) != XP_OK)
        return s;
    (*out)->load_info = info;
    (*out)->load_from_cache = from_cache ? 1 : 0;
    (*out)->load_cache_written = written ? 1 : 0;
    return XP_OK;
}

xp_status xp_session_load_info(xp_session* s, int* from_cache, int* cache_written, char* msg, uint32_t msg_bytes) {
    if (!s) return xp::fail(XP_ERR_INVALID, "xp_session_load_info: null session");
    if (from_cache) *from_cache = s->load_from_cache;
    if (cache_written) *cache_written = s->load_cache_written;
    if (msg && msg_bytes) std::snprintf(msg, msg_bytes, "%s", s->load_info.c_str());
    return XP_OK;
}

xp_status xp_session_config(xp_session* s, xp_model_config* cfg) {
    if (!s || !cfg) return xp::fail(XP_ERR_INVALID, "xp_session_config: null argument");
    *cfg = s->cfg;
    return XP_OK;
}

}  // extern "C"
