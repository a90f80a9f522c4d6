// Checkpoint -> resident registry: colizig_cuda_moe_load_safetensors.
//
// The reference's host opens every safetensors shard, indexes the tensors by
// name from the shard headers (src/model/manifest.zig, weights.zig:198-235) and
// loads one routed expert at a time from the mmap into its LRU
// (src/qwen38/moe.zig:251-292 loadExpert, 306-329 Layer.load).  Here a whole MoE
// layer goes from the mapped shards into resident device memory in one call:
// the headers are parsed (a small JSON reader, bounds-checked: the files are
// inputs), the shards are mapped read-only, and the tensors' bytes are handed to
// colizig_cuda_moe_register_layer as host pointers, which copies them to the
// device.  Names follow the reference: `<prefix>.<suffix>` first, then the bare
// suffix (weights.zig viewBySuffix), with suffixes
//   layers.L.mlp.gate.weight                              router [E, H]  F32 | BF16
//   layers.L.mlp.experts.e.{gate,up,down}_proj.weight      E4M3 [I, H] / [H, I]
//   layers.L.mlp.experts.e.{gate,up,down}_proj.weight_scale_inv   [nblk, nblk] F32 | BF16 | F16
//   layers.L.mlp.shared_expert.{gate,up,down}_proj.weight(_scale_inv), shared_expert_gate.weight
//   (a BF16 shared expert, as real Qwen4-Exp checkpoints hold it, has no _scale_inv)
// BF16 / F16 values are widened exactly to f32 (bf16: the top 16 bits of an
// f32, as matmul.zig:105-107 bf16ToF32), which is what the reference's dotBf16
// multiplies by, so a BF16 router gives the same logits as its f32 widening.
#include <fcntl.h>
#include <stdint.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cuda_fp16.h>

#include <map>
#include <string>
#include <vector>

#include "../../include/colizig_cuda.h"
#include "cz_common.cuh"

#define CZ_EXPORT extern "C" __attribute__((visibility("default")))

namespace {

struct StTensor {
    std::string dtype;
    std::vector<uint64_t> shape;
    uint64_t begin = 0, end = 0;  // offsets in the shard's data section
};

// A minimal JSON reader for safetensors headers: objects, arrays, strings,
// unsigned integers; other values are skipped.  Every read is bounds-checked.
struct Json {
    const char* p;
    const char* e;
    int depth = 0;
    void ws() {
        while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
    }
    bool eat(char c) {
        ws();
        if (p < e && *p == c) {
            ++p;
            return true;
        }
        return false;
    }
    bool str(std::string& out) {
        ws();
        if (p >= e || *p != '"') return false;
        ++p;
        out.clear();
        while (p < e && *p != '"') {
            if (*p == '\\') {
                if (++p >= e) return false;
                const char c = *p;
                if (c == 'u') {  // keep \uXXXX as written: tensor names are ASCII in practice
                    if (e - p < 5) return false;
                    out.append(p - 1, 6);
                    p += 5;
                    continue;
                }
                out.push_back(c == 'n' ? '\n' : c == 't' ? '\t' : c);
                ++p;
                continue;
            }
            out.push_back(*p++);
        }
        if (p >= e) return false;
        ++p;
        return true;
    }
    bool uint(uint64_t& v) {
        ws();
        if (p >= e || *p < '0' || *p > '9') return false;
        v = 0;
        while (p < e && *p >= '0' && *p <= '9') {
            if (v > (UINT64_MAX - 9) / 10) return false;
            v = v * 10 + (uint64_t)(*p++ - '0');
        }
        return true;
    }
    bool skip() {  // any value
        ws();
        if (p >= e || ++depth > 64) return false;
        bool ok = true;
        if (*p == '"') {
            std::string s;
            ok = str(s);
        } else if (*p == '{' || *p == '[') {
            const char close = *p == '{' ? '}' : ']';
            const bool obj = *p == '{';
            ++p;
            if (!eat(close)) {
                do {
                    if (obj) {
                        std::string k;
                        ok = str(k) && eat(':');
                    }
                    ok = ok && skip();
                } while (ok && eat(','));
                ok = ok && eat(close);
            }
        } else {
            while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
        }
        --depth;
        return ok;
    }
    bool uint_array(std::vector<uint64_t>& out) {
        out.clear();
        if (!eat('[')) return false;
        if (eat(']')) return true;
        do {
            uint64_t v;
            if (!uint(v)) return false;
            out.push_back(v);
        } while (eat(','));
        return eat(']');
    }
    bool tensor(StTensor& t) {
        if (!eat('{')) return false;
        if (eat('}')) return false;
        bool have_off = false;
        do {
            std::string k;
            if (!str(k) || !eat(':')) return false;
            if (k == "dtype") {
                if (!str(t.dtype)) return false;
            } else if (k == "shape") {
                if (!uint_array(t.shape)) return false;
            } else if (k == "data_offsets") {
                std::vector<uint64_t> o;
                if (!uint_array(o) || o.size() != 2 || o[1] < o[0]) return false;
                t.begin = o[0];
                t.end = o[1];
                have_off = true;
            } else if (!skip()) {
                return false;
            }
        } while (eat(','));
        return eat('}') && have_off && !t.dtype.empty();
    }
    bool header(std::map<std::string, StTensor>& out) {
        if (!eat('{')) return false;
        if (eat('}')) return true;
        do {
            std::string name;
            if (!str(name) || !eat(':')) return false;
            if (name == "__metadata__") {
                if (!skip()) return false;
                continue;
            }
            StTensor t;
            if (!tensor(t)) return false;
            out[name] = t;
        } while (eat(','));
        return eat('}');
    }
};

size_t elem_size(const std::string& dt) {
    if (dt == "F8_E4M3" || dt == "U8" || dt == "I8") return 1;
    if (dt == "BF16" || dt == "F16") return 2;
    if (dt == "F32") return 4;
    return 0;
}

struct Shard {
    int fd = -1;
    const uint8_t* map = nullptr;
    size_t size = 0, data0 = 0;
    std::map<std::string, StTensor> index;
    ~Shard() {
        if (map) munmap(const_cast<uint8_t*>(map), size);
        if (fd >= 0) close(fd);
    }
};

constexpr int CZ_EIO = -10;

// Opens and indexes one shard (the header), and maps the whole file read-only.
int open_shard(const char* path, Shard& s) {
    s.fd = open(path, O_RDONLY);
    if (s.fd < 0) return CZ_EIO;
    struct stat st;
    if (fstat(s.fd, &st) != 0 || st.st_size < 8) return CZ_EIO;
    s.size = (size_t)st.st_size;
    void* m = mmap(nullptr, s.size, PROT_READ, MAP_PRIVATE, s.fd, 0);
    if (m == MAP_FAILED) return CZ_EIO;
    s.map = static_cast<const uint8_t*>(m);
    uint64_t n = 0;
    for (int i = 0; i < 8; ++i) n |= (uint64_t)s.map[i] << (8 * i);
    // header cap as the reference's (safetensors.zig:23 max_header_bytes, checked at :139)
    if (n == 0 || n > s.size - 8 || n > (256ull << 20)) return CZ_EIO;
    s.data0 = 8 + (size_t)n;
    Json j{reinterpret_cast<const char*>(s.map) + 8, reinterpret_cast<const char*>(s.map) + 8 + n};
    if (!j.header(s.index)) return CZ_EIO;
    for (auto& kv : s.index) {  // every tensor lies inside the file and has the bytes its shape says
        const StTensor& t = kv.second;
        if (t.end > s.size - s.data0) return CZ_EIO;
        const size_t es = elem_size(t.dtype);
        if (es) {
            uint64_t numel = 1;
            for (uint64_t d : t.shape) {
                if (d && numel > UINT64_MAX / d) return CZ_EIO;
                numel *= d;
            }
            if (numel * es != t.end - t.begin) return CZ_EIO;
        }
    }
    return CZ_OK;
}

struct View {
    const StTensor* t = nullptr;
    const uint8_t* bytes = nullptr;
};

struct Index {
    std::vector<Shard> shards;
    std::string prefix;
    // <prefix>.<suffix>, then the bare suffix (weights.zig viewBySuffix)
    View find(const std::string& suffix) const {
        for (int pass = 0; pass < 2; ++pass) {
            if (pass == 0 && prefix.empty()) continue;
            const std::string name = pass == 0 ? prefix + "." + suffix : suffix;
            for (const Shard& s : shards) {
                auto it = s.index.find(name);
                if (it != s.index.end()) return View{&it->second, s.map + s.data0 + it->second.begin};
            }
        }
        return View{};
    }
};

bool shape_is(const StTensor& t, std::initializer_list<uint64_t> want) {
    return t.shape.size() == want.size() && std::equal(want.begin(), want.end(), t.shape.begin());
}

// f32 values of a F32 / BF16 / F16 tensor: the mapped bytes themselves for F32,
// else an exact widening into `keep` (which owns the storage).
const float* as_f32(const View& v, std::vector<std::vector<float>>& keep) {
    const StTensor& t = *v.t;
    const size_t n = (t.end - t.begin) / elem_size(t.dtype);
    if (t.dtype == "F32") {
        if ((reinterpret_cast<uintptr_t>(v.bytes) & 3u) == 0) return reinterpret_cast<const float*>(v.bytes);
        keep.emplace_back(n);
        memcpy(keep.back().data(), v.bytes, n * 4);
        return keep.back().data();
    }
    keep.emplace_back(n);
    float* out = keep.back().data();
    for (size_t i = 0; i < n; ++i) {
        uint16_t b;
        memcpy(&b, v.bytes + 2 * i, 2);
        if (t.dtype == "BF16") {
            const uint32_t w = (uint32_t)b << 16;
            memcpy(&out[i], &w, 4);
        } else {
            out[i] = __half2float(__ushort_as_half(b));
        }
    }
    return out;
}

bool is_float(const StTensor& t) { return t.dtype == "F32" || t.dtype == "BF16" || t.dtype == "F16"; }

size_t nblk(uint64_t x) { return (size_t)((x + 127) / 128); }

}  // namespace

CZ_EXPORT int colizig_cuda_moe_load_safetensors(uint32_t layer, const char* const* shard_paths, int n_shards,
                                                const char* prefix, uint32_t layer_index,
                                                const colizig_moe_dims* dims, uint32_t flags) {
    if (!shard_paths || n_shards < 1 || !dims || (flags & COLIZIG_PTR_DEVICE)) return CZ_EARGS;
    const colizig_moe_dims d = *dims;
    if (d.hidden == 0 || d.experts == 0 || d.inter == 0) return CZ_EARGS;
    Index ix;
    ix.prefix = prefix ? prefix : "";
    ix.shards.resize((size_t)n_shards);
    for (int i = 0; i < n_shards; ++i) {
        if (!shard_paths[i]) return CZ_EARGS;
        const int rc = open_shard(shard_paths[i], ix.shards[(size_t)i]);
        if (rc) return rc;
    }
    const uint64_t H = d.hidden, I = d.inter, SI = d.shared_inter, E = d.experts;
    const std::string L = "layers." + std::to_string(layer_index) + ".mlp.";
    std::vector<std::vector<float>> keep;

    const View router = ix.find(L + "gate.weight");
    if (!router.t) return CZ_EIO;
    if (!is_float(*router.t) || !shape_is(*router.t, {E, H})) return CZ_ESHAPE;
    const float* router_f = as_f32(router, keep);

    // one block-FP8 projection: E4M3 [rows, cols] + scales [nblk(rows), nblk(cols)]
    auto fp8 = [&](const std::string& stem, uint64_t rows, uint64_t cols, const uint8_t** w,
                   const float** sc) -> int {
        const View wv = ix.find(stem + ".weight"), sv = ix.find(stem + ".weight_scale_inv");
        if (!wv.t || !sv.t) return CZ_EIO;
        if (wv.t->dtype != "F8_E4M3" || !shape_is(*wv.t, {rows, cols})) return CZ_ESHAPE;
        if (!is_float(*sv.t) || !shape_is(*sv.t, {nblk(rows), nblk(cols)})) return CZ_ESHAPE;
        *w = wv.bytes;
        *sc = as_f32(sv, keep);
        return CZ_OK;
    };
    std::vector<colizig_moe_expert> ex(E);
    for (uint64_t e = 0; e < E; ++e) {
        const std::string stem = L + "experts." + std::to_string(e) + ".";
        colizig_moe_expert& x = ex[e];
        int rc = fp8(stem + "gate_proj", I, H, &x.gate_w, &x.gate_s);
        if (!rc) rc = fp8(stem + "up_proj", I, H, &x.up_w, &x.up_s);
        if (!rc) rc = fp8(stem + "down_proj", H, I, &x.down_w, &x.down_s);
        if (rc) return rc;
    }
    colizig_moe_expert sh{};
    const float* sh_gate = nullptr;
    uint32_t sh_flag = 0;
    if (SI) {
        const std::string stem = L + "shared_expert.";
        const View g0 = ix.find(stem + "gate_proj.weight");
        if (g0.t && g0.t->dtype == "BF16") {
            // the reference's BF16 NativeMatrix shared expert (moe.zig:319-325,
            // tensors.zig:74-95): bf16 [SI, H] gate/up, [H, SI] down, no scales
            const View u0 = ix.find(stem + "up_proj.weight"), dn = ix.find(stem + "down_proj.weight");
            if (!u0.t || !dn.t) return CZ_EIO;
            if (u0.t->dtype != "BF16" || dn.t->dtype != "BF16" || !shape_is(*g0.t, {SI, H}) ||
                !shape_is(*u0.t, {SI, H}) || !shape_is(*dn.t, {H, SI}))
                return CZ_ESHAPE;
            sh.gate_w = g0.bytes;
            sh.up_w = u0.bytes;
            sh.down_w = dn.bytes;
            sh_flag = COLIZIG_SHARED_BF16;
        } else {
            int rc = fp8(stem + "gate_proj", SI, H, &sh.gate_w, &sh.gate_s);
            if (!rc) rc = fp8(stem + "up_proj", SI, H, &sh.up_w, &sh.up_s);
            if (!rc) rc = fp8(stem + "down_proj", H, SI, &sh.down_w, &sh.down_s);
            if (rc) return rc;
        }
        const View g = ix.find(L + "shared_expert_gate.weight");
        if (!g.t) return CZ_EIO;
        if (!is_float(*g.t) || !(shape_is(*g.t, {H}) || shape_is(*g.t, {1, H}))) return CZ_ESHAPE;
        sh_gate = as_f32(g, keep);
    }
    return colizig_cuda_moe_register_layer(layer, &d, router_f, ex.data(), SI ? &sh : nullptr, sh_gate,
                                           (flags & COLIZIG_EP) | sh_flag);
}
