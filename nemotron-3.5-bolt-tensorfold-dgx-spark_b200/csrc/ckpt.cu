// Checkpoint ingestion: the model's safetensors shards, memory-mapped, looked up by tensor name and packed into this
// engine's device layouts.  It replaces libbolt's Store / open_store / lookup and the loaders around them
// (bolt_host.cu:61-345: load_slab, load_nv4, load_q8), for the weights of this path:
//   model.safetensors.index.json   {"weight_map": {tensor name: shard file}}  (or one model.safetensors, no index)
//   each shard                     8-byte little-endian header length N, a JSON header of N bytes
//                                  {name: {"dtype": .., "shape": [..], "data_offsets": [begin, end]}, "__metadata__": ..},
//                                  then the data, the offsets counted from its start.
// The header is read by a small JSON parser of its own (objects, arrays, strings with escapes, numbers, literals),
// which checks every offset against the file before a tensor is handed out.  Shards are mapped on first use.  The
// packers copy each tensor's raw bytes (host, from the mapping) into a caller-owned device staging buffer and run the
// engine's packer from there, all on the caller's stream; they validate names, byte counts and staging sizes before
// the first copy.
#include "common.cuh"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <initializer_list>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace b200q {
namespace {

// ---------------------------------------------------------------------------------------------------------
// JSON (RFC 8259), enough of it for safetensors headers and the shard index
// ---------------------------------------------------------------------------------------------------------
struct JVal {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0;
    bool is_uint = false;   // a number written as a plain non-negative integer, kept exactly in u
    uint64_t u = 0;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;

    const JVal* get(const char* key) const {
        if (kind != Obj) return nullptr;
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class JParser {
  public:
    JParser(const char* p, size_t n) : p_(p), e_(p + n) {}
    bool parse(JVal& v) {
        ws();
        if (!value(v, 0)) return false;
        ws();
        return p_ == e_ || all_padding();
    }

  private:
    const char* p_;
    const char* e_;
    static constexpr int kMaxDepth = 64;

    bool all_padding() {   // safetensors pads its header with spaces; NULs are tolerated too
        for (; p_ < e_; p_++)
            if (*p_ != ' ' && *p_ != '\0') return false;
        return true;
    }
    void ws() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) p_++;
    }
    bool lit(const char* s) {
        const size_t n = strlen(s);
        if ((size_t)(e_ - p_) < n || memcmp(p_, s, n) != 0) return false;
        p_ += n;
        return true;
    }
    static void utf8(std::string& out, uint32_t cp) {
        if (cp < 0x80) out += (char)cp;
        else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 63)); }
        else if (cp < 0x10000) {
            out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 63)); out += (char)(0x80 | (cp & 63));
        } else {
            out += (char)(0xF0 | (cp >> 18)); out += (char)(0x80 | ((cp >> 12) & 63));
            out += (char)(0x80 | ((cp >> 6) & 63)); out += (char)(0x80 | (cp & 63));
        }
    }
    bool hex4(uint32_t& v) {
        if (e_ - p_ < 4) return false;
        v = 0;
        for (int i = 0; i < 4; i++) {
            const char c = *p_++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else return false;
        }
        return true;
    }
    bool string(std::string& out) {
        if (p_ >= e_ || *p_ != '"') return false;
        p_++;
        while (p_ < e_) {
            const char c = *p_++;
            if (c == '"') return true;
            if ((unsigned char)c < 0x20) return false;
            if (c != '\\') { out += c; continue; }
            if (p_ >= e_) return false;
            const char x = *p_++;
            switch (x) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t cp;
                    if (!hex4(cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {   // a surrogate pair
                        uint32_t lo;
                        if (!lit("\\u") || !hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return false;
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp < 0xE000) {
                        return false;
                    }
                    utf8(out, cp);
                    break;
                }
                default: return false;
            }
        }
        return false;
    }
    bool number(JVal& v) {
        const char* s = p_;
        if (p_ < e_ && *p_ == '-') p_++;
        if (p_ >= e_ || !(*p_ >= '0' && *p_ <= '9')) return false;
        if (*p_ == '0') p_++;
        else while (p_ < e_ && *p_ >= '0' && *p_ <= '9') p_++;
        bool integer = *s != '-';
        if (p_ < e_ && *p_ == '.') {
            integer = false;
            p_++;
            if (p_ >= e_ || !(*p_ >= '0' && *p_ <= '9')) return false;
            while (p_ < e_ && *p_ >= '0' && *p_ <= '9') p_++;
        }
        if (p_ < e_ && (*p_ == 'e' || *p_ == 'E')) {
            integer = false;
            p_++;
            if (p_ < e_ && (*p_ == '+' || *p_ == '-')) p_++;
            if (p_ >= e_ || !(*p_ >= '0' && *p_ <= '9')) return false;
            while (p_ < e_ && *p_ >= '0' && *p_ <= '9') p_++;
        }
        const std::string tok(s, p_);
        v.kind = JVal::Num;
        v.num = strtod(tok.c_str(), nullptr);
        if (integer && tok.size() <= 19) {   // below 10^19: no u64 overflow
            v.is_uint = true;
            v.u = strtoull(tok.c_str(), nullptr, 10);
        }
        return true;
    }
    bool value(JVal& v, int depth) {
        if (depth > kMaxDepth || p_ >= e_) return false;
        const char c = *p_;
        if (c == '{') {
            p_++;
            v.kind = JVal::Obj;
            ws();
            if (p_ < e_ && *p_ == '}') { p_++; return true; }
            while (true) {
                ws();
                std::pair<std::string, JVal> kv;
                if (!string(kv.first)) return false;
                ws();
                if (p_ >= e_ || *p_++ != ':') return false;
                ws();
                if (!value(kv.second, depth + 1)) return false;
                v.obj.push_back(std::move(kv));
                ws();
                if (p_ >= e_) return false;
                if (*p_ == ',') { p_++; continue; }
                if (*p_ == '}') { p_++; return true; }
                return false;
            }
        }
        if (c == '[') {
            p_++;
            v.kind = JVal::Arr;
            ws();
            if (p_ < e_ && *p_ == ']') { p_++; return true; }
            while (true) {
                ws();
                JVal x;
                if (!value(x, depth + 1)) return false;
                v.arr.push_back(std::move(x));
                ws();
                if (p_ >= e_) return false;
                if (*p_ == ',') { p_++; continue; }
                if (*p_ == ']') { p_++; return true; }
                return false;
            }
        }
        if (c == '"') { v.kind = JVal::Str; return string(v.str); }
        if (c == 't') { v.kind = JVal::Bool; v.b = true; return lit("true"); }
        if (c == 'f') { v.kind = JVal::Bool; v.b = false; return lit("false"); }
        if (c == 'n') { v.kind = JVal::Null; return lit("null"); }
        return number(v);
    }
};

// ---------------------------------------------------------------------------------------------------------
// the store
// ---------------------------------------------------------------------------------------------------------
struct Tensor {
    std::string dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;   // from the start of the shard's data
};

struct Shard {
    const uint8_t* base = nullptr;
    size_t size = 0;
    uint64_t data0 = 0;            // 8 + header length
    bool tried = false, ok = false;
    std::unordered_map<std::string, Tensor> tensors;
};

// bytes an element of a safetensors dtype (0: unknown, not checked)
size_t dtype_bytes(const std::string& d) {
    if (d == "U8" || d == "I8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
    if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
    if (d == "F32" || d == "I32" || d == "U32") return 4;
    if (d == "F64" || d == "I64" || d == "U64") return 8;
    return 0;
}

bool read_file(const std::string& path, std::string& out) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return false;
    std::string s;
    char buf[65536];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) s.append(buf, n);
    const bool err = ferror(f) != 0;
    fclose(f);
    if (err) return false;
    out.swap(s);
    return true;
}

// a shard file name from the index: relative, without parent references
bool safe_name(const std::string& f) {
    if (f.empty() || f[0] == '/') return false;
    size_t i = 0;
    while (i <= f.size()) {
        const size_t j = f.find('/', i);
        const std::string part = f.substr(i, j == std::string::npos ? std::string::npos : j - i);
        if (part.empty() || part == "..") return false;
        if (j == std::string::npos) break;
        i = j + 1;
    }
    return true;
}

bool parse_header(Shard& sh) {
    if (sh.size < 8) return false;
    uint64_t n = 0;
    for (int i = 7; i >= 0; i--) n = (n << 8) | sh.base[i];   // little-endian
    if (n > sh.size - 8) return false;
    JVal h;
    if (!JParser(reinterpret_cast<const char*>(sh.base) + 8, (size_t)n).parse(h) || h.kind != JVal::Obj) return false;
    sh.data0 = 8 + n;
    const uint64_t avail = sh.size - sh.data0;
    for (const auto& kv : h.obj) {
        if (kv.first == "__metadata__") continue;
        const JVal& t = kv.second;
        const JVal *dt = t.get("dtype"), *shp = t.get("shape"), *off = t.get("data_offsets");
        if (!dt || dt->kind != JVal::Str || !shp || shp->kind != JVal::Arr || !off || off->kind != JVal::Arr ||
            off->arr.size() != 2 || !off->arr[0].is_uint || !off->arr[1].is_uint)
            return false;
        Tensor x;
        x.dtype = dt->str;
        x.begin = off->arr[0].u;
        x.end = off->arr[1].u;
        if (x.begin > x.end || x.end > avail) return false;
        uint64_t numel = 1;
        for (const JVal& d : shp->arr) {
            if (!d.is_uint || d.u > (1ull << 40)) return false;
            x.shape.push_back((int64_t)d.u);
            numel *= d.u;
            if (numel > (1ull << 50)) return false;
        }
        const size_t eb = dtype_bytes(x.dtype);
        if (eb && numel * eb != x.end - x.begin) return false;
        sh.tensors.emplace(kv.first, std::move(x));
    }
    return true;
}

}  // namespace

struct Ckpt {
    std::string dir;
    std::unordered_map<std::string, std::string> shard_of;   // tensor name -> shard file
    std::unordered_map<std::string, Shard> shards;
    std::mutex mu;

    ~Ckpt() {
        for (auto& kv : shards)
            if (kv.second.base) munmap(const_cast<uint8_t*>(kv.second.base), kv.second.size);
    }

    Shard* open_shard(const std::string& file) {
        Shard& sh = shards[file];
        if (sh.tried) return sh.ok ? &sh : nullptr;
        sh.tried = true;
        const std::string path = dir + "/" + file;
        const int fd = open(path.c_str(), O_RDONLY);
        if (fd < 0) return nullptr;
        struct stat st;
        if (fstat(fd, &st) != 0 || st.st_size < 8) {
            close(fd);
            return nullptr;
        }
        void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
        close(fd);
        if (m == MAP_FAILED) return nullptr;
        sh.base = static_cast<const uint8_t*>(m);
        sh.size = (size_t)st.st_size;
        sh.ok = parse_header(sh);
        return sh.ok ? &sh : nullptr;
    }

    // the tensor and its bytes in the mapping, or null
    const Tensor* find(const std::string& name, const uint8_t** data) {
        std::lock_guard<std::mutex> lock(mu);
        const auto it = shard_of.find(name);
        if (it == shard_of.end()) return nullptr;
        Shard* sh = open_shard(it->second);
        if (!sh) return nullptr;
        const auto jt = sh->tensors.find(name);
        if (jt == sh->tensors.end()) return nullptr;
        *data = sh->base + sh->data0 + jt->second.begin;
        return &jt->second;
    }
};

}  // namespace b200q

using namespace b200q;

struct b200q_ckpt : Ckpt {};

namespace {

// a tensor of exactly `bytes` bytes and, when `shape` is given, exactly that shape, or null.  The byte count alone
// would accept a tensor whose rows and k are swapped (the same count, another layout); the reference's loaders read n
// and k from the shape and check its last dimension (load_iq2 / load_q8 / load_nv4, engine/bolt_host.cu:198-283).
const Tensor* sized(b200q_ckpt* c, const std::string& name, size_t bytes, const uint8_t** data,
                    std::initializer_list<int64_t> shape = {}) {
    const Tensor* t = c->find(name, data);
    if (!t || t->end - t->begin != bytes) return nullptr;
    if (shape.size() && (t->shape.size() != shape.size() || !std::equal(shape.begin(), shape.end(), t->shape.begin())))
        return nullptr;
    return t;
}

inline size_t up16(size_t v) { return (v + 15) & ~size_t(15); }

int h2d(void* dst, const void* src, size_t bytes, void* stream) {
    return status_from(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream));
}

}  // namespace

extern "C" {

b200q_ckpt* b200q_ckpt_open(const char* dir) {
    if (!dir) return nullptr;
    std::unique_ptr<b200q_ckpt> c(new b200q_ckpt());
    c->dir = dir;
    std::string idx;
    if (read_file(c->dir + "/model.safetensors.index.json", idx)) {
        JVal j;
        if (!JParser(idx.data(), idx.size()).parse(j)) return nullptr;
        const JVal* wm = j.get("weight_map");
        if (!wm || wm->kind != JVal::Obj) return nullptr;
        for (const auto& kv : wm->obj) {
            if (kv.second.kind != JVal::Str || !safe_name(kv.second.str)) return nullptr;
            c->shard_of[kv.first] = kv.second.str;
        }
        return c.release();
    }
    // one file and no index: every tensor of model.safetensors
    Shard* sh = c->open_shard("model.safetensors");
    if (!sh) return nullptr;
    for (const auto& kv : sh->tensors) c->shard_of[kv.first] = "model.safetensors";
    return c.release();
}

void b200q_ckpt_close(b200q_ckpt* c) { delete c; }

int64_t b200q_ckpt_count(b200q_ckpt* c) { return c ? (int64_t)c->shard_of.size() : -1; }

int b200q_ckpt_tensor(b200q_ckpt* c, const char* name, const void** data, size_t* bytes, int64_t* shape, int* ndim,
                      char* dtype) {
    if (!c || !name) return B200Q_EINVAL;
    const uint8_t* p = nullptr;
    const Tensor* t = c->find(name, &p);
    if (!t || t->shape.size() > 8 || t->dtype.size() > 15) return B200Q_EINVAL;
    if (data) *data = p;
    if (bytes) *bytes = (size_t)(t->end - t->begin);
    if (ndim) *ndim = (int)t->shape.size();
    if (shape)
        for (size_t i = 0; i < t->shape.size(); i++) shape[i] = t->shape[i];
    if (dtype) snprintf(dtype, 16, "%s", t->dtype.c_str());
    return B200Q_OK;
}

size_t b200q_ckpt_staging_bytes(int fmt, int n, int k) {
    if (n <= 0 || k <= 0) return 0;
    if (fmt == 0) return (size_t)n * (k / 256) * 66;                                 // one expert's IQ2_XXS blocks
    if (fmt == 1) return up16((size_t)n * (k / 2)) + (size_t)n * (k / 16);          // NVFP4 codes, then scales
    if (fmt == 2) return (size_t)n * (k / 32) * 34;                                  // Q8_0 blocks
    return 0;
}

int b200q_ckpt_pack_iq2_slab(b200q_ckpt* c, const char* const* names, int experts, int rows, int k, void* packed,
                             void* staging, size_t staging_bytes, void* stream) {
    if (!c || !names || experts <= 0 || rows <= 0 || rows % 32 || k <= 0 || k % 256 || !packed || !staging ||
        ((uintptr_t)staging & 15) || ((uintptr_t)packed & 15))
        return B200Q_EINVAL;
    const size_t raw = b200q_ckpt_staging_bytes(0, rows, k);
    if (staging_bytes < raw) return B200Q_ENOSPACE;
    std::vector<const uint8_t*> src((size_t)experts);
    for (int e = 0; e < experts; e++)   // every expert found and of the right size before the first copy
        if (!names[e] || !sized(c, names[e], raw, &src[(size_t)e], {rows, k / 256, 66})) return B200Q_EINVAL;
    const size_t per = iq2_bytes(rows, k);
    for (int e = 0; e < experts; e++) {
        int st = h2d(staging, src[(size_t)e], raw, stream);
        if (st == B200Q_OK) st = b200q_iq2_pack(staging, (uint8_t*)packed + (size_t)e * per, rows, k, stream);
        if (st != B200Q_OK) return st;
    }
    return B200Q_OK;
}

int b200q_ckpt_pack_nv4(b200q_ckpt* c, const char* prefix, int n, int k, void* packed, float* s2, void* staging,
                        size_t staging_bytes, void* stream) {
    if (!c || !prefix || n <= 0 || n % 16 || k <= 0 || k % 256 || !packed || !s2 || !staging || ((uintptr_t)staging & 15))
        return B200Q_EINVAL;
    if (staging_bytes < b200q_ckpt_staging_bytes(1, n, k)) return B200Q_ENOSPACE;
    const std::string p(prefix);
    const uint8_t *q = nullptr, *sc = nullptr, *g = nullptr;
    const size_t qb = (size_t)n * (k / 2), sb = (size_t)n * (k / 16);
    if (!sized(c, p + ".weight", qb, &q, {n, k / 2}) || !sized(c, p + ".weight_scale", sb, &sc, {n, k / 16}) ||
        !sized(c, p + ".weight_scale_2", 4, &g))
        return B200Q_EINVAL;
    memcpy(s2, g, 4);
    uint8_t* st8 = static_cast<uint8_t*>(staging);
    int st = h2d(st8, q, qb, stream);
    if (st == B200Q_OK) st = h2d(st8 + up16(qb), sc, sb, stream);
    if (st == B200Q_OK) st = b200q_nv4_pack(st8, st8 + up16(qb), packed, n, k, stream);
    return st;
}

int b200q_ckpt_pack_q8(b200q_ckpt* c, const char* name, int n, int k, void* packed, void* staging,
                       size_t staging_bytes, void* stream) {
    if (!c || !name || n <= 0 || n % 16 || k <= 0 || k % 256 || !packed || !staging || ((uintptr_t)staging & 15))
        return B200Q_EINVAL;
    const size_t raw = b200q_ckpt_staging_bytes(2, n, k);
    if (staging_bytes < raw) return B200Q_ENOSPACE;
    const uint8_t* src = nullptr;
    if (!sized(c, name, raw, &src, {n, k / 32, 34})) return B200Q_EINVAL;
    int st = h2d(staging, src, raw, stream);
    if (st == B200Q_OK) st = b200q_q8_pack(staging, packed, n, k, stream);
    return st;
}

}  // extern "C"
