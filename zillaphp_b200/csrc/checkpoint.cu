// checkpoint.cu -- the net's flat parameter (and Adam state) buffers as a
// SafeTensors F32 file in the reference's checkpoint layout:
//   [8 bytes]  header size, u64 little-endian
//   [H bytes]  JSON header, compact, padded with spaces to a multiple of 8
//   [D bytes]  the tensors' F32 data, concatenated in header order
// with one tensor "param_i" per parameter in Module::parameters() order
// ([W, b] per Conv2D / Linear; the Transformer LM's list as zilla_lm_create
// documents it), exactly as ModelSerializer::save writes a model through
// SafeTensorsSerializer::save (src/Serialization/ModelSerializer.php:56-69,
// src/Serialization/SafeTensorsSerializer.php:32-98).  The reference stores
// only the parameters; with_state adds the Adam moments as "adam_m_i" /
// "adam_v_i" (same shapes) and the step count as __metadata__ "adam_t".
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <string>
#include <vector>

#include "net.cuh"

namespace zb {

int lm_param_shapes(Net &n, std::vector<std::vector<long long>> &shapes);   // lm_net.cu

namespace {

// Shapes of the net's parameter tensors in order (their sizes tile the flat buffer).
int param_shapes(Net &n, std::vector<std::vector<long long>> &shapes) {
    shapes.clear();
    if (n.lm) return lm_param_shapes(n, shapes);
    for (const Stage &s : n.st) {
        if (s.kind == kConv) {
            shapes.push_back({s.oC, s.C, 3, 3});
            shapes.push_back({s.oC});
        } else if (s.kind == kLinear) {
            shapes.push_back({s.in_n, s.oC});
            shapes.push_back({s.oC});
        }
    }
    return kOk;
}

long long numel(const std::vector<long long> &s) {
    long long k = 1;
    for (long long d : s) k *= d;
    return k;
}

// ---- a small JSON reader for SafeTensors headers (objects, arrays, strings, numbers)
struct Json {
    const char *p, *e;
    void ws() { while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
    bool lit(char c) { ws(); if (p < e && *p == c) { ++p; return true; } return false; }
    bool str(std::string &out) {
        ws();
        if (p >= e || *p != '"') return false;
        ++p;
        out.clear();
        while (p < e && *p != '"') {
            if (*p == '\\') {   // escapes: keep the escaped character (names are plain ASCII)
                if (++p >= e) return false;
                if (*p == 'u') { if (e - p < 5) return false; out += '?'; p += 5; continue; }
            }
            out += *p++;
        }
        if (p >= e) return false;
        ++p;
        return true;
    }
    bool num(long long &v) {
        ws();
        const char *q = p;
        bool neg = false;
        if (q < e && *q == '-') { neg = true; ++q; }
        if (q >= e || *q < '0' || *q > '9') return false;
        long long x = 0;
        while (q < e && *q >= '0' && *q <= '9') x = x * 10 + (*q++ - '0');
        p = q;
        v = neg ? -x : x;
        return true;
    }
    bool ints(std::vector<long long> &out) {
        out.clear();
        if (!lit('[')) return false;
        if (lit(']')) return true;
        do {
            long long v;
            if (!num(v)) return false;
            out.push_back(v);
        } while (lit(','));
        return lit(']');
    }
    bool skip() {   // any value
        ws();
        if (p >= e) return false;
        if (*p == '"') { std::string s; return str(s); }
        if (*p == '{' || *p == '[') {
            const char open = *p, close = open == '{' ? '}' : ']';
            ++p;
            if (lit(close)) return true;
            do {
                if (open == '{') { std::string k; if (!str(k) || !lit(':')) return false; }
                if (!skip()) return false;
            } while (lit(','));
            return lit(close);
        }
        while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;   // number / true / false / null
        return true;
    }
};

struct Entry {
    std::string name, dtype;
    std::vector<long long> shape, offs;
};

bool parse_header(const char *p, const char *e, std::vector<Entry> &out, std::string &adam_t) {
    Json j{p, e};
    if (!j.lit('{')) return false;
    if (j.lit('}')) return true;
    do {
        std::string key;
        if (!j.str(key) || !j.lit(':')) return false;
        if (key == "__metadata__") {
            if (!j.lit('{')) return false;
            if (j.lit('}')) continue;
            do {
                std::string k, v;
                if (!j.str(k) || !j.lit(':') || !j.str(v)) return false;   // values are strings
                if (k == "adam_t") adam_t = v;
            } while (j.lit(','));
            if (!j.lit('}')) return false;
            continue;
        }
        Entry en;
        en.name = key;
        if (!j.lit('{')) return false;
        if (!j.lit('}')) {
            do {
                std::string f;
                if (!j.str(f) || !j.lit(':')) return false;
                if (f == "dtype") { if (!j.str(en.dtype)) return false; }
                else if (f == "shape") { if (!j.ints(en.shape)) return false; }
                else if (f == "data_offsets") { if (!j.ints(en.offs) || en.offs.size() != 2) return false; }
                else if (!j.skip()) return false;
            } while (j.lit(','));
            if (!j.lit('}')) return false;
        }
        out.push_back(en);
    } while (j.lit(','));
    return j.lit('}');
}

std::string shape_json(const std::vector<long long> &s) {
    std::string o = "[";
    for (size_t i = 0; i < s.size(); ++i) o += (i ? "," : "") + std::to_string(s[i]);
    return o + "]";
}

}  // namespace

}  // namespace zb

using namespace zb;

extern "C" {

int zilla_net_save(int id, const char *path, int with_state) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_save: unknown net %d", id);
    if (!path) return fail(kBadArg, "zilla_net_save: null path");
    if (with_state && n->peer.on)
        return fail(kBadArg, "zilla_net_save: the Adam state is sliced over the data-parallel ranks; detach first");
    std::vector<std::vector<long long>> shapes;
    int rc = param_shapes(*n, shapes);
    if (rc) return rc;
    long long total = 0;
    for (auto &s : shapes) total += numel(s);
    if (total != n->nparams) return fail(kBadArg, "zilla_net_save: parameter shapes do not tile the buffer");
    std::vector<float> host((size_t)n->nparams * (with_state ? 3 : 1));
    cudaStreamSynchronize(stream());
    if (cudaMemcpy(host.data(), n->params, (size_t)n->nparams * 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
        (with_state && (cudaMemcpy(host.data() + n->nparams, n->m, (size_t)n->nparams * 4, cudaMemcpyDeviceToHost) !=
                            cudaSuccess ||
                        cudaMemcpy(host.data() + 2 * n->nparams, n->v, (size_t)n->nparams * 4,
                                   cudaMemcpyDeviceToHost) != cudaSuccess)))
        return check_cuda("zilla_net_save: download");
    // header: param_i, then (with_state) adam_m_i, adam_v_i; offsets in bytes
    std::string h = "{";
    long long off = 0;
    const char *prefix[3] = {"param_", "adam_m_", "adam_v_"};
    for (int part = 0; part < (with_state ? 3 : 1); ++part)
        for (size_t i = 0; i < shapes.size(); ++i) {
            const long long bytes = numel(shapes[i]) * 4;
            if (h.size() > 1) h += ",";
            h += "\"" + std::string(prefix[part]) + std::to_string(i) + "\":{\"dtype\":\"F32\",\"shape\":" +
                 shape_json(shapes[i]) + ",\"data_offsets\":[" + std::to_string(off) + "," +
                 std::to_string(off + bytes) + "]}";
            off += bytes;
        }
    if (with_state) h += ",\"__metadata__\":{\"adam_t\":\"" + std::to_string(n->t) + "\"}";
    h += "}";
    while (h.size() % 8) h += ' ';
    FILE *f = fopen(path, "wb");
    if (!f) return fail(kBadArg, "zilla_net_save: cannot open %s", path);
    const unsigned long long hs = h.size();
    unsigned char le[8];
    for (int i = 0; i < 8; ++i) le[i] = (unsigned char)(hs >> (8 * i));
    bool ok = fwrite(le, 1, 8, f) == 8 && fwrite(h.data(), 1, h.size(), f) == h.size() &&
              fwrite(host.data(), 4, host.size(), f) == host.size();
    ok = (fclose(f) == 0) && ok;
    return ok ? kOk : fail(kBadArg, "zilla_net_save: write to %s failed", path);
}

int zilla_net_load(int id, const char *path) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_load: unknown net %d", id);
    if (!path) return fail(kBadArg, "zilla_net_load: null path");
    // attached over peer memory, the ranks' parameters are identical by construction and each
    // rank holds only its slice of the Adam state: a load on some ranks would break both
    if (n->peer.on)
        return fail(kBadArg, "zilla_net_load: the net is attached for data parallelism over peer memory; "
                             "detach first, load the same file on every rank, then attach");
    FILE *f = fopen(path, "rb");
    if (!f) return fail(kBadArg, "zilla_net_load: checkpoint not found: %s", path);
    std::vector<char> raw;
    {
        char buf[1 << 16];
        size_t k;
        while ((k = fread(buf, 1, sizeof(buf), f)) > 0) raw.insert(raw.end(), buf, buf + k);
        fclose(f);
    }
    if (raw.size() < 8) return fail(kBadArg, "zilla_net_load: file too small to be a SafeTensors file");
    unsigned long long hs = 0;
    for (int i = 0; i < 8; ++i) hs |= (unsigned long long)(unsigned char)raw[i] << (8 * i);
    if (hs > raw.size() - 8) return fail(kBadArg, "zilla_net_load: truncated SafeTensors file");
    std::vector<Entry> ents;
    std::string adam_t;
    if (!parse_header(raw.data() + 8, raw.data() + 8 + hs, ents, adam_t))
        return fail(kBadArg, "zilla_net_load: invalid SafeTensors header");
    const size_t data0 = 8 + (size_t)hs;
    std::vector<std::vector<long long>> shapes;
    int rc = param_shapes(*n, shapes);
    if (rc) return rc;
    // every tensor this net needs: param_i (required), adam_m_i / adam_v_i (all or none)
    auto find = [&](const std::string &name) -> const Entry * {
        for (const Entry &en : ents) if (en.name == name) return &en;
        return nullptr;
    };
    auto check = [&](const Entry *en, size_t i) -> int {
        if (en->dtype != "F32")
            return fail(kBadArg, "zilla_net_load: only F32 is supported (got '%s' for '%s')", en->dtype.c_str(),
                        en->name.c_str());
        if (en->shape != shapes[i]) return fail(kBadArg, "zilla_net_load: shape mismatch for '%s'", en->name.c_str());
        if (en->offs[0] < 0 || en->offs[1] - en->offs[0] != numel(shapes[i]) * 4 ||
            data0 + (size_t)en->offs[1] > raw.size())
            return fail(kBadArg, "zilla_net_load: bad data offsets for '%s'", en->name.c_str());
        return kOk;
    };
    std::vector<float> host[3];
    int parts = 1;
    for (int part = 0; part < 3; ++part) {
        const char *prefix = part == 0 ? "param_" : part == 1 ? "adam_m_" : "adam_v_";
        if (part > 0 && !find(std::string(prefix) + "0")) break;
        host[part].resize((size_t)n->nparams);
        long long off = 0;
        for (size_t i = 0; i < shapes.size(); ++i) {
            const std::string name = std::string(prefix) + std::to_string(i);
            const Entry *en = find(name);
            if (!en) return fail(kBadArg, "zilla_net_load: missing parameter '%s' in checkpoint", name.c_str());
            if ((rc = check(en, i))) return rc;
            memcpy(host[part].data() + off, raw.data() + data0 + en->offs[0], (size_t)numel(shapes[i]) * 4);
            off += numel(shapes[i]);
        }
        parts = part + 1;
    }
    if (parts == 2) return fail(kBadArg, "zilla_net_load: adam_m_* without adam_v_*");
    cudaStreamSynchronize(stream());
    if (cudaMemcpy(n->params, host[0].data(), (size_t)n->nparams * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return check_cuda("zilla_net_load: upload");
    if (parts == 3) {
        if (cudaMemcpy(n->m, host[1].data(), (size_t)n->nparams * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(n->v, host[2].data(), (size_t)n->nparams * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return check_cuda("zilla_net_load: upload of the Adam state");
        if (!adam_t.empty()) n->t = atoi(adam_t.c_str());
    }
    return check_cuda("zilla_net_load");
}

}  // extern "C"
