// Host-only parts of the C ABI: version / status strings, device count, the
// safetensors reader (include/safetensors.h:23-53 of the reference, extended
// with BF16), and the checkpoint loaders that map the reference's tensor
// names (src/utils/dit_loader.cpp:47-115, src/utils/patchenc_loader.cpp:175-208)
// onto the engine weight structs.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "runtime.h"

struct dtts_st {
    FILE *fp = nullptr;
    uint64_t data_start = 0;
    struct Info {
        std::string dtype;
        std::vector<int64_t> shape;
        uint64_t begin = 0, end = 0;
    };
    std::map<std::string, Info> tensors;
    ~dtts_st() {
        if (fp) fclose(fp);
    }
};

namespace {

// ---- minimal JSON reader for the safetensors header -----------------------
struct Json {
    const char *p, *end;
    void ws() { while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++; }
    bool eat(char c) { ws(); if (p < end && *p == c) { p++; return true; } return false; }
    bool str(std::string &out) {
        ws();
        if (p >= end || *p != '"') return false;
        p++;
        out.clear();
        while (p < end && *p != '"') {
            if (*p == '\\' && p + 1 < end) { out.push_back(p[1]); p += 2; continue; }
            out.push_back(*p++);
        }
        if (p >= end) return false;
        p++;
        return true;
    }
    bool num(int64_t &v) {
        ws();
        char *e = nullptr;
        v = strtoll(p, &e, 10);
        if (e == p) return false;
        p = e;
        return true;
    }
    // skips any JSON value (used for __metadata__)
    bool skip() {
        ws();
        if (p >= end) return false;
        if (*p == '"') { std::string s; return str(s); }
        if (*p == '{' || *p == '[') {
            const char open = *p, close = open == '{' ? '}' : ']';
            int depth = 0;
            bool in_str = false;
            for (; p < end; p++) {
                if (in_str) { if (*p == '\\') p++; else if (*p == '"') in_str = false; continue; }
                if (*p == '"') in_str = true;
                else if (*p == open) depth++;
                else if (*p == close && --depth == 0) { p++; return true; }
            }
            return false;
        }
        while (p < end && *p != ',' && *p != '}' && *p != ']') p++;
        return true;
    }
};

float half_to_f32(uint16_t h) {
    const uint32_t s = (h >> 15) & 1, e = (h >> 10) & 0x1f, m = h & 0x3ff;
    uint32_t u;
    if (e == 0) {
        if (m == 0) u = s << 31;
        else {  // subnormal
            int ee = -1;
            uint32_t mm = m;
            do { ee++; mm <<= 1; } while ((mm & 0x400) == 0);
            u = (s << 31) | ((uint32_t)(127 - 15 - ee) << 23) | ((mm & 0x3ff) << 13);
        }
    } else if (e == 31) {
        u = (s << 31) | 0x7f800000u | (m << 13);
    } else {
        u = (s << 31) | ((e - 15 + 127) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

}  // namespace

extern "C" {

const char *dtts_version(void) { return "dtts-b200 0.1 (sm_100a)"; }

const char *dtts_status_string(int s) {
    switch (s) {
        case DTTS_OK: return "ok";
        case DTTS_ERR_ARG: return "invalid argument";
        case DTTS_ERR_CUDA: return "CUDA error";
        case DTTS_ERR_OOM: return "out of device memory";
        case DTTS_ERR_TIMEOUT: return "timed out";
        case DTTS_ERR_NONFINITE: return "non-finite result";
        case DTTS_ERR_UNSUPPORTED: return "unsupported";
        case DTTS_ERR_IO: return "I/O or format error";
        case DTTS_ERR_NO_DEVICE: return "no usable device";
    }
    return "unknown status";
}

const char *dtts_last_error(void) { return dtts::last_error(); }

int dtts_fp8_quantize_rows(const float *w, int rows, int cols, uint8_t *q, float *scale) {
    DTTS_CHECK(w && q && scale && rows >= 1 && cols >= 1, DTTS_ERR_ARG, "bad fp8 quantisation arguments");
    dtts::e4m3_quantize_rows(w, (size_t)rows, (size_t)cols, q, scale, nullptr);
    return DTTS_OK;
}

int dtts_device_count(int *n) {
    if (!n) return DTTS_ERR_ARG;
    *n = 0;
    int c = 0;
    if (cudaGetDeviceCount(&c) != cudaSuccess) { cudaGetLastError(); return DTTS_OK; }
    for (int d = 0; d < c; d++) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, d) == cudaSuccess && p.major == 10) (*n)++;
    }
    return DTTS_OK;
}

int dtts_st_open(const char *path, dtts_st **out) {
    using dtts::set_error;
    if (!path || !out) { set_error("null argument"); return DTTS_ERR_ARG; }
    *out = nullptr;
    std::unique_ptr<dtts_st> f(new dtts_st());
    f->fp = fopen(path, "rb");
    if (!f->fp) { set_error("cannot open %s", path); return DTTS_ERR_IO; }
    uint64_t hl = 0;
    if (fread(&hl, 8, 1, f->fp) != 1 || hl == 0 || hl > (uint64_t)1 << 30) { set_error("%s: bad header length", path); return DTTS_ERR_IO; }
    std::string hdr(hl, '\0');
    if (fread(&hdr[0], 1, hl, f->fp) != hl) { set_error("%s: truncated header", path); return DTTS_ERR_IO; }
    f->data_start = 8 + hl;
    fseeko(f->fp, 0, SEEK_END);
    const uint64_t fsize = (uint64_t)ftello(f->fp);
    Json j{hdr.data(), hdr.data() + hdr.size()};
    if (!j.eat('{')) { set_error("%s: header is not a JSON object", path); return DTTS_ERR_IO; }
    if (!j.eat('}')) {
        do {
            std::string name;
            if (!j.str(name) || !j.eat(':')) { set_error("%s: malformed header", path); return DTTS_ERR_IO; }
            if (name == "__metadata__") { if (!j.skip()) { set_error("%s: malformed metadata", path); return DTTS_ERR_IO; } continue; }
            dtts_st::Info info;
            if (!j.eat('{')) { set_error("%s: malformed entry %s", path, name.c_str()); return DTTS_ERR_IO; }
            bool have_off = false;
            do {
                std::string key;
                if (!j.str(key) || !j.eat(':')) { set_error("%s: malformed entry %s", path, name.c_str()); return DTTS_ERR_IO; }
                if (key == "dtype") {
                    if (!j.str(info.dtype)) { set_error("%s: bad dtype", path); return DTTS_ERR_IO; }
                } else if (key == "shape") {
                    if (!j.eat('[')) { set_error("%s: bad shape", path); return DTTS_ERR_IO; }
                    if (!j.eat(']')) {
                        do { int64_t v; if (!j.num(v)) { set_error("%s: bad shape", path); return DTTS_ERR_IO; } info.shape.push_back(v); } while (j.eat(','));
                        if (!j.eat(']')) { set_error("%s: bad shape", path); return DTTS_ERR_IO; }
                    }
                } else if (key == "data_offsets") {
                    int64_t a, b;
                    if (!j.eat('[') || !j.num(a) || !j.eat(',') || !j.num(b) || !j.eat(']')) { set_error("%s: bad offsets", path); return DTTS_ERR_IO; }
                    info.begin = (uint64_t)a; info.end = (uint64_t)b; have_off = true;
                } else if (!j.skip()) { set_error("%s: malformed entry", path); return DTTS_ERR_IO; }
            } while (j.eat(','));
            if (!j.eat('}') || !have_off || info.end < info.begin || f->data_start + info.end > fsize) {
                set_error("%s: tensor %s has bad offsets", path, name.c_str());
                return DTTS_ERR_IO;
            }
            f->tensors[name] = info;
        } while (j.eat(','));
        if (!j.eat('}')) { set_error("%s: malformed header end", path); return DTTS_ERR_IO; }
    }
    *out = f.release();
    return DTTS_OK;
}

int dtts_st_close(dtts_st *f) {
    delete f;
    return DTTS_OK;
}

int dtts_st_count(dtts_st *f, int *n) {
    if (!f || !n) return DTTS_ERR_ARG;
    *n = (int)f->tensors.size();
    return DTTS_OK;
}

int dtts_st_shape(dtts_st *f, const char *name, int *ndim, int64_t *shape) {
    if (!f || !name || !ndim) return DTTS_ERR_ARG;
    auto it = f->tensors.find(name);
    if (it == f->tensors.end()) { dtts::set_error("tensor %s not found", name); return DTTS_ERR_IO; }
    *ndim = (int)it->second.shape.size();
    if (shape)
        for (size_t i = 0; i < it->second.shape.size() && i < 8; i++) shape[i] = it->second.shape[i];
    return DTTS_OK;
}

int dtts_st_read_f32(dtts_st *f, const char *name, float *dst, size_t n) {
    using dtts::set_error;
    if (!f || !name || !dst) return DTTS_ERR_ARG;
    auto it = f->tensors.find(name);
    if (it == f->tensors.end()) { set_error("tensor %s not found", name); return DTTS_ERR_IO; }
    const dtts_st::Info &in = it->second;
    size_t count = 1;
    for (int64_t d : in.shape) count *= (size_t)d;
    if (count != n) { set_error("tensor %s has %zu elements, caller expects %zu", name, count, n); return DTTS_ERR_ARG; }
    const size_t esz = in.dtype == "F32" ? 4 : (in.dtype == "F16" || in.dtype == "BF16") ? 2 : 0;
    if (!esz) { set_error("tensor %s: dtype %s not supported (F32, F16, BF16)", name, in.dtype.c_str()); return DTTS_ERR_UNSUPPORTED; }
    if (in.end - in.begin != count * esz) { set_error("tensor %s: byte size mismatch", name); return DTTS_ERR_IO; }
    fseeko(f->fp, (off_t)(f->data_start + in.begin), SEEK_SET);
    if (esz == 4) {
        if (fread(dst, 4, count, f->fp) != count) { set_error("tensor %s: short read", name); return DTTS_ERR_IO; }
        return DTTS_OK;
    }
    std::vector<uint16_t> tmp(count);
    if (fread(tmp.data(), 2, count, f->fp) != count) { set_error("tensor %s: short read", name); return DTTS_ERR_IO; }
    if (in.dtype == "F16") {
        for (size_t i = 0; i < count; i++) dst[i] = half_to_f32(tmp[i]);
    } else {
        for (size_t i = 0; i < count; i++) { uint32_t u = (uint32_t)tmp[i] << 16; std::memcpy(&dst[i], &u, 4); }
    }
    return DTTS_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ loaders
namespace {

struct HostTensors {
    std::vector<std::vector<float>> store;
    const float *get(dtts_st *f, const std::string &name, size_t n, bool required, int *st) {
        int nd = 0;
        int64_t shp[8];
        if (dtts_st_shape(f, name.c_str(), &nd, shp) != DTTS_OK) {
            if (required) { dtts::set_error("checkpoint lacks %s", name.c_str()); *st = DTTS_ERR_IO; }
            return nullptr;
        }
        store.emplace_back(n);
        int r = dtts_st_read_f32(f, name.c_str(), store.back().data(), n);
        if (r) { *st = r; return nullptr; }
        return store.back().data();
    }
};

}  // namespace

extern "C" {

int dtts_dit_create_from_safetensors(const char *path, int n_layers, int dtype, int device, dtts_dit **out) {
    if (!out) return DTTS_ERR_ARG;
    if (n_layers <= 0) n_layers = 18;
    dtts_st *f = nullptr;
    int st = dtts_st_open(path, &f);
    if (st) return st;
    std::unique_ptr<dtts_st> guard(f);
    HostTensors H;
    std::vector<dtts_dit_block_weights> blocks(n_layers);
    const size_t D = 1024, F = 4096;
    for (int i = 0; i < n_layers; i++) {
        const std::string p = "velocity_field_predictor.blocks." + std::to_string(i) + ".";
        dtts_dit_block_weights &b = blocks[i];
        b.wq = H.get(f, p + "attn.q_proj.weight", D * D, true, &st);
        b.wk = H.get(f, p + "attn.k_proj.weight", D * D, true, &st);
        b.wv = H.get(f, p + "attn.v_proj.weight", D * D, true, &st);
        b.wo = H.get(f, p + "attn.o_proj.weight", D * D, true, &st);
        b.bo = H.get(f, p + "attn.o_proj.bias", D, false, &st);
        b.qn = H.get(f, p + "attn.q_norm.weight", 64, false, &st);
        b.kn = H.get(f, p + "attn.k_norm.weight", 64, false, &st);
        b.w1 = H.get(f, p + "ffn.fc1.weight", F * D, true, &st);
        b.b1 = H.get(f, p + "ffn.fc1.bias", F, false, &st);
        b.w2 = H.get(f, p + "ffn.fc2.weight", D * F, true, &st);
        b.b2 = H.get(f, p + "ffn.fc2.bias", D, false, &st);
        b.ada_w = H.get(f, p + "adaLN_modulation.1.weight", 6 * D * D, true, &st);
        b.ada_b = H.get(f, p + "adaLN_modulation.1.bias", 6 * D, false, &st);
        if (st) return st;
    }
    dtts_dit_weights w;
    std::memset(&w, 0, sizeof(w));
    w.n_layers = n_layers;
    w.blocks = blocks.data();
    const std::string v = "velocity_field_predictor.";
    w.t_w1 = H.get(f, v + "time_embedder.mlp.0.weight", D * 256, true, &st);
    w.t_b1 = H.get(f, v + "time_embedder.mlp.0.bias", D, false, &st);
    w.t_w2 = H.get(f, v + "time_embedder.mlp.2.weight", D * D, true, &st);
    w.t_b2 = H.get(f, v + "time_embedder.mlp.2.bias", D, false, &st);
    w.spk_w1 = H.get(f, "xvec_proj.0.weight", D * 512, false, &st);
    w.spk_b1 = H.get(f, "xvec_proj.0.bias", D, false, &st);
    w.spk_ln_w = H.get(f, "xvec_proj.1.weight", D, false, &st);
    w.spk_ln_b = H.get(f, "xvec_proj.1.bias", D, false, &st);
    w.oada_w = H.get(f, v + "output_layer.adaLN_modulation.1.weight", 2 * D * D, true, &st);
    w.oada_b = H.get(f, v + "output_layer.adaLN_modulation.1.bias", 2 * D, false, &st);
    w.out_w = H.get(f, v + "output_layer.linear.weight", 128 * D, true, &st);
    w.out_b = H.get(f, v + "output_layer.linear.bias", 128, false, &st);
    w.in_w = H.get(f, v + "input_layer.weight", D * D, true, &st);
    w.in_b = H.get(f, v + "input_layer.bias", D, false, &st);
    w.hid_w = H.get(f, "hidden_proj.weight", D * 1536, false, &st);
    w.hid_b = H.get(f, "hidden_proj.bias", D, false, &st);
    w.lat_w = H.get(f, "latent_proj.weight", D * 128, false, &st);
    w.lat_b = H.get(f, "latent_proj.bias", D, false, &st);
    w.coord_w = H.get(f, "coordinate_proj.weight", D * 128, true, &st);
    w.coord_b = H.get(f, "coordinate_proj.bias", D, false, &st);
    w.eos_w1 = H.get(f, "eos_proj.0.weight", 1536 * 1536, false, &st);   // src/utils/dit_loader.cpp:109-112
    w.eos_b1 = H.get(f, "eos_proj.0.bias", 1536, false, &st);
    w.eos_w2 = H.get(f, "eos_proj.2.weight", 2 * 1536, false, &st);
    w.eos_b2 = H.get(f, "eos_proj.2.bias", 2, false, &st);
    if (st) return st;
    return dtts_dit_create(&w, dtype, device, out);
}

int dtts_pe_create_from_safetensors(const char *path, int n_layers, int dtype, int device, int max_batch,
                                    int max_tokens, dtts_pe **out) {
    if (!out) return DTTS_ERR_ARG;
    if (n_layers <= 0) n_layers = 24;
    dtts_st *f = nullptr;
    int st = dtts_st_open(path, &f);
    if (st) return st;
    std::unique_ptr<dtts_st> guard(f);
    HostTensors H;
    std::vector<dtts_pe_layer_weights> layers(n_layers);
    const size_t D = 1024, F = 4096;
    for (int i = 0; i < n_layers; i++) {
        const std::string p = "patch_encoder.encoder.layers." + std::to_string(i) + ".";
        dtts_pe_layer_weights &l = layers[i];
        l.wq = H.get(f, p + "attn.q_proj.weight", D * D, true, &st);
        l.wk = H.get(f, p + "attn.k_proj.weight", D * D, true, &st);
        l.wv = H.get(f, p + "attn.v_proj.weight", D * D, true, &st);
        l.wo = H.get(f, p + "attn.o_proj.weight", D * D, true, &st);
        l.bo = H.get(f, p + "attn.o_proj.bias", D, false, &st);
        l.attn_norm_w = H.get(f, p + "attn_norm.weight", D, false, &st);
        l.w1 = H.get(f, p + "ffn.fc1.weight", F * D, true, &st);
        l.b1 = H.get(f, p + "ffn.fc1.bias", F, false, &st);
        l.w2 = H.get(f, p + "ffn.fc2.weight", D * F, true, &st);
        l.b2 = H.get(f, p + "ffn.fc2.bias", D, false, &st);
        l.ffn_norm_w = H.get(f, p + "ffn_norm.weight", D, false, &st);
        if (st) return st;
    }
    dtts_pe_weights w;
    std::memset(&w, 0, sizeof(w));
    w.n_layers = n_layers;
    w.layers = layers.data();
    w.conv_w = H.get(f, "patch_encoder.ds_proj.weight", 128 * 128 * 2, true, &st);
    w.conv_b = H.get(f, "patch_encoder.ds_proj.bias", 128, false, &st);
    w.in_w = H.get(f, "patch_encoder.in_proj.weight", D * 128, true, &st);
    w.in_b = H.get(f, "patch_encoder.in_proj.bias", D, false, &st);
    w.out_w = H.get(f, "patch_encoder.out_proj.weight", 1536 * 2 * D, true, &st);
    w.out_b = H.get(f, "patch_encoder.out_proj.bias", 1536, false, &st);
    if (st) return st;
    return dtts_pe_create(&w, dtype, device, max_batch, max_tokens, out);
}

}  // extern "C"
