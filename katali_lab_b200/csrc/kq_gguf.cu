// kq_gguf.cu — GGUF container reader and native-layout device upload (katali_cuda_gguf_*).
//
// The reference's engine reads GGUF files with its own parser (V/src/gguf_reader.c:351-545,
// V/include/katali_gguf.h:64-152) and hands tensor bytes to its backends in their native
// block layout (V/src/gguf_model.c:187-227). Here the same container is parsed on the host
// from a read-only memory mapping, every read bounds-checked, and a tensor's bytes go to
// device memory unchanged (GGUF super-blocks are the kernels' layout) through two pinned
// staging buffers: the CPU copy of chunk i + 1 out of the mapping overlaps the DMA of
// chunk i on the plugin stream.
//
// Container (GGUF v2/v3, little-endian): magic "GGUF", u32 version, u64 tensor count,
// u64 metadata count; metadata entries (string key, u32 value type, value; arrays carry
// an element type and u64 count and may not nest); tensor entries (string name, u32 n_dims,
// u64 dims[n_dims] with dims[0] contiguous, u32 ggml type, u64 offset); the data section
// starts at the next multiple of general.alignment (default 32) and every tensor offset is
// relative to it and aligned to it.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <string>
#include <vector>

#include "katali_cuda.h"

namespace kq {
int ensure_runtime();
void set_status_message(const char *msg);
cudaStream_t current_stream();
void dense_adopt_weights(KataliDense *m, void *mem);
void hybrid_adopt(KataliHybrid *m, std::vector<void *> allocs, std::vector<KataliMoe *> moes,
                  std::vector<void *> pinned, KataliExpertCache *cache);
}  // namespace kq

namespace {

constexpr uint32_t GGUF_MAGIC = 0x46554747u;  // "GGUF"
enum : uint32_t {
    V_U8 = 0, V_I8 = 1, V_U16 = 2, V_I16 = 3, V_U32 = 4, V_I32 = 5, V_F32 = 6, V_BOOL = 7,
    V_STR = 8, V_ARR = 9, V_U64 = 10, V_I64 = 11, V_F64 = 12
};
constexpr uint64_t MAX_STR = 1ull << 30;
constexpr uint32_t MAX_DIMS = 4;
constexpr size_t STAGE = 32u << 20;  // bytes per pinned staging buffer

// Elements per block and bytes per block of the ggml types this reader sizes; 0: unknown.
void type_block(uint32_t t, uint64_t &per, uint64_t &bytes) {
    per = 1;
    switch (t) {
        case 0: bytes = 4; return;    // F32
        case 1: bytes = 2; return;    // F16
        case 2: per = 32; bytes = 18; return;    // Q4_0
        case 3: per = 32; bytes = 20; return;    // Q4_1
        case 6: per = 32; bytes = 22; return;    // Q5_0
        case 7: per = 32; bytes = 24; return;    // Q5_1
        case 8: per = 32; bytes = 34; return;    // Q8_0
        case 9: per = 32; bytes = 36; return;    // Q8_1
        case 10: per = 256; bytes = 84; return;  // Q2_K
        case 11: per = 256; bytes = 110; return; // Q3_K
        case 12: per = 256; bytes = 144; return; // Q4_K
        case 13: per = 256; bytes = 176; return; // Q5_K
        case 14: per = 256; bytes = 210; return; // Q6_K
        case 15: per = 256; bytes = 292; return; // Q8_K
        case 24: bytes = 1; return;   // I8
        case 25: bytes = 2; return;   // I16
        case 26: bytes = 4; return;   // I32
        case 27: bytes = 8; return;   // I64
        case 28: bytes = 8; return;   // F64
        case 30: bytes = 2; return;   // BF16
        default: bytes = 0; return;
    }
}

struct Kv {
    std::string key;
    uint32_t type = 0, elem = 0;  // elem: array element type
    uint64_t count = 0;           // array length
    uint64_t pos = 0;             // file offset of the value (array: of its first element)
};

struct Tensor {
    std::string name;
    uint32_t n_dims = 0, type = 0;
    uint64_t dims[MAX_DIMS] = {1, 1, 1, 1};
    uint64_t rel = 0, abs = 0, nbytes = 0;
};

struct Cursor {
    const uint8_t *p;
    uint64_t size, at;
    bool ok = true;
    bool need(uint64_t n) {
        if (!ok || n > size - at) ok = false;
        return ok;
    }
    template <typename T>
    T get() {
        T v{};
        if (need(sizeof(T))) {
            memcpy(&v, p + at, sizeof(T));
            at += sizeof(T);
        }
        return v;
    }
    bool str(std::string *out) {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > MAX_STR || !need(n)) return ok = false;
        if (out) out->assign(reinterpret_cast<const char *>(p + at), (size_t)n);
        at += n;
        return true;
    }
};

uint64_t scalar_size(uint32_t t) {
    switch (t) {
        case V_U8: case V_I8: case V_BOOL: return 1;
        case V_U16: case V_I16: return 2;
        case V_U32: case V_I32: case V_F32: return 4;
        case V_U64: case V_I64: case V_F64: return 8;
        default: return 0;
    }
}

}  // namespace

struct KataliGguf {
    int fd = -1;
    const uint8_t *map = nullptr;
    uint64_t size = 0;
    uint32_t version = 0;
    uint64_t alignment = 32, data_off = 0;
    std::vector<Kv> kv;
    std::vector<Tensor> t;
    void *stage[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
};

namespace {

int fail(KataliGguf *g, const char *why) {
    kq::set_status_message(why);
    if (g) katali_cuda_gguf_close(g);
    return KATALI_ERR_BAD_ARG;
}

const Kv *find_kv(const KataliGguf *g, const char *key) {
    for (const Kv &k : g->kv)
        if (k.key == key) return &k;
    return nullptr;
}

bool read_scalar(const KataliGguf *g, const Kv &k, uint32_t type, uint64_t pos, int64_t *iv, double *fv) {
    const uint8_t *q = g->map + pos;
    switch (type) {
        case V_U8: *iv = q[0]; break;
        case V_I8: *iv = (int8_t)q[0]; break;
        case V_BOOL: *iv = q[0] != 0; break;
        case V_U16: { uint16_t v; memcpy(&v, q, 2); *iv = v; break; }
        case V_I16: { int16_t v; memcpy(&v, q, 2); *iv = v; break; }
        case V_U32: { uint32_t v; memcpy(&v, q, 4); *iv = v; break; }
        case V_I32: { int32_t v; memcpy(&v, q, 4); *iv = v; break; }
        case V_U64: { uint64_t v; memcpy(&v, q, 8); *iv = (int64_t)v; break; }
        case V_I64: { int64_t v; memcpy(&v, q, 8); *iv = v; break; }
        case V_F32: { float v; memcpy(&v, q, 4); *fv = v; return true; }
        case V_F64: { double v; memcpy(&v, q, 8); *fv = v; return true; }
        default: return false;
    }
    *fv = (double)*iv;
    (void)k;
    return true;
}

}  // namespace

extern "C" {

int katali_cuda_gguf_open(const char *path, KataliGguf **out) {
    if (!path || !out) return KATALI_ERR_BAD_ARG;
    *out = nullptr;
    KataliGguf *g = new KataliGguf();
    g->fd = open(path, O_RDONLY | O_CLOEXEC);
    if (g->fd < 0) return fail(g, "katali_cuda_gguf_open: cannot open the file");
    struct stat st;
    if (fstat(g->fd, &st) != 0 || st.st_size < 24) return fail(g, "katali_cuda_gguf_open: not a GGUF file (too short)");
    g->size = (uint64_t)st.st_size;
    void *m = mmap(nullptr, (size_t)g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (m == MAP_FAILED) return fail(g, "katali_cuda_gguf_open: mmap failed");
    g->map = (const uint8_t *)m;
    Cursor c{g->map, g->size, 0};
    if (c.get<uint32_t>() != GGUF_MAGIC) return fail(g, "katali_cuda_gguf_open: bad magic");
    g->version = c.get<uint32_t>();
    if (g->version != 2 && g->version != 3) return fail(g, "katali_cuda_gguf_open: unsupported GGUF version");
    const uint64_t nt = c.get<uint64_t>(), nkv = c.get<uint64_t>();
    // every entry needs at least 8 (string length) + 4 bytes: bounds the counts
    if (!c.ok || nt > g->size / 12 || nkv > g->size / 12) return fail(g, "katali_cuda_gguf_open: bad counts");
    g->kv.resize((size_t)nkv);
    for (Kv &k : g->kv) {
        if (!c.str(&k.key)) return fail(g, "katali_cuda_gguf_open: truncated metadata key");
        k.type = c.get<uint32_t>();
        if (!c.ok) return fail(g, "katali_cuda_gguf_open: truncated metadata");
        if (k.type == V_STR) {
            k.pos = c.at;
            if (!c.str(nullptr)) return fail(g, "katali_cuda_gguf_open: truncated string value");
        } else if (k.type == V_ARR) {
            k.elem = c.get<uint32_t>();
            k.count = c.get<uint64_t>();
            if (!c.ok) return fail(g, "katali_cuda_gguf_open: truncated array");
            if (k.elem == V_ARR) return fail(g, "katali_cuda_gguf_open: nested metadata array");
            k.pos = c.at;
            if (k.elem == V_STR) {
                if (k.count > (g->size - c.at) / 8) return fail(g, "katali_cuda_gguf_open: bad array length");
                for (uint64_t i = 0; i < k.count; ++i)
                    if (!c.str(nullptr)) return fail(g, "katali_cuda_gguf_open: truncated string array");
            } else {
                const uint64_t es = scalar_size(k.elem);
                if (!es) return fail(g, "katali_cuda_gguf_open: bad array element type");
                if (k.count > (g->size - c.at) / es || !c.need(k.count * es))
                    return fail(g, "katali_cuda_gguf_open: truncated array");
                c.at += k.count * es;
            }
        } else {
            const uint64_t es = scalar_size(k.type);
            if (!es) return fail(g, "katali_cuda_gguf_open: bad metadata value type");
            k.pos = c.at;
            if (!c.need(es)) return fail(g, "katali_cuda_gguf_open: truncated metadata value");
            c.at += es;
        }
    }
    if (const Kv *a = find_kv(g, "general.alignment")) {
        int64_t iv = 0;
        double fv = 0;
        if (a->type == V_ARR || a->type == V_STR || !read_scalar(g, *a, a->type, a->pos, &iv, &fv) ||
            iv <= 0 || (iv & (iv - 1)) != 0)
            return fail(g, "katali_cuda_gguf_open: bad general.alignment");
        g->alignment = (uint64_t)iv;
    }
    g->t.resize((size_t)nt);
    for (Tensor &t : g->t) {
        if (!c.str(&t.name)) return fail(g, "katali_cuda_gguf_open: truncated tensor name");
        t.n_dims = c.get<uint32_t>();
        if (!c.ok || t.n_dims == 0 || t.n_dims > MAX_DIMS) return fail(g, "katali_cuda_gguf_open: bad tensor rank");
        for (uint32_t d = 0; d < t.n_dims; ++d) t.dims[d] = c.get<uint64_t>();
        t.type = c.get<uint32_t>();
        t.rel = c.get<uint64_t>();
        if (!c.ok) return fail(g, "katali_cuda_gguf_open: truncated tensor entry");
    }
    g->data_off = (c.at + g->alignment - 1) / g->alignment * g->alignment;
    if (g->data_off > g->size) return fail(g, "katali_cuda_gguf_open: truncated before the data section");
    for (Tensor &t : g->t) {
        uint64_t n = 1;
        for (uint32_t d = 0; d < t.n_dims; ++d) {
            if (t.dims[d] == 0 || n > UINT64_MAX / t.dims[d]) return fail(g, "katali_cuda_gguf_open: bad tensor dims");
            n *= t.dims[d];
        }
        if (t.rel % g->alignment) return fail(g, "katali_cuda_gguf_open: misaligned tensor offset");
        uint64_t per, bytes;
        type_block(t.type, per, bytes);
        if (bytes && t.dims[0] % per == 0) {
            const uint64_t rb = t.dims[0] / per * bytes;
            if (n / t.dims[0] > UINT64_MAX / rb) return fail(g, "katali_cuda_gguf_open: tensor too large");
            t.nbytes = rb * (n / t.dims[0]);
        }
        if (t.rel > g->size - g->data_off || t.nbytes > g->size - g->data_off - t.rel)
            return fail(g, "katali_cuda_gguf_open: tensor data out of range");
        t.abs = g->data_off + t.rel;
    }
    *out = g;
    return KATALI_OK;
}

int katali_cuda_gguf_close(KataliGguf *g) {
    if (!g) return KATALI_OK;
    for (int i = 0; i < 2; ++i) {
        if (g->done[i]) {
            cudaEventSynchronize(g->done[i]);
            cudaEventDestroy(g->done[i]);
        }
        if (g->stage[i]) cudaFreeHost(g->stage[i]);
    }
    if (g->map) munmap((void *)g->map, (size_t)g->size);
    if (g->fd >= 0) close(g->fd);
    delete g;
    return KATALI_OK;
}

int katali_cuda_gguf_counts(const KataliGguf *g, uint64_t *n_tensors, uint64_t *n_kv, uint32_t *version) {
    if (!g) return KATALI_ERR_BAD_ARG;
    if (n_tensors) *n_tensors = g->t.size();
    if (n_kv) *n_kv = g->kv.size();
    if (version) *version = g->version;
    return KATALI_OK;
}

int katali_cuda_gguf_tensor(const KataliGguf *g, uint64_t i, KataliGgufTensorInfo *info) {
    if (!g || !info || i >= g->t.size()) return KATALI_ERR_BAD_ARG;
    const Tensor &t = g->t[(size_t)i];
    info->name = t.name.c_str();
    info->type = t.type;
    info->n_dims = t.n_dims;
    for (uint32_t d = 0; d < 4; ++d) info->dims[d] = t.dims[d];
    info->offset = t.abs;
    info->nbytes = t.nbytes;
    return KATALI_OK;
}

int katali_cuda_gguf_find(const KataliGguf *g, const char *name, uint64_t *index) {
    if (!g || !name || !index) return KATALI_ERR_BAD_ARG;
    for (size_t i = 0; i < g->t.size(); ++i)
        if (g->t[i].name == name) {
            *index = i;
            return KATALI_OK;
        }
    kq::set_status_message("katali_cuda_gguf_find: no tensor of that name");
    return KATALI_ERR_BAD_ARG;
}

int katali_cuda_gguf_get_int(const KataliGguf *g, const char *key, int64_t *v) {
    if (!g || !key || !v) return KATALI_ERR_BAD_ARG;
    const Kv *k = find_kv(g, key);
    double fv = 0;
    if (!k || k->type == V_ARR || k->type == V_STR || k->type == V_F32 || k->type == V_F64 ||
        !read_scalar(g, *k, k->type, k->pos, v, &fv))
        return KATALI_ERR_BAD_ARG;
    return KATALI_OK;
}

int katali_cuda_gguf_get_float(const KataliGguf *g, const char *key, double *v) {
    if (!g || !key || !v) return KATALI_ERR_BAD_ARG;
    const Kv *k = find_kv(g, key);
    int64_t iv = 0;
    if (!k || k->type == V_ARR || k->type == V_STR || !read_scalar(g, *k, k->type, k->pos, &iv, v))
        return KATALI_ERR_BAD_ARG;
    return KATALI_OK;
}

int katali_cuda_gguf_get_str(const KataliGguf *g, const char *key, const char **s, uint64_t *len) {
    if (!g || !key || !s) return KATALI_ERR_BAD_ARG;
    const Kv *k = find_kv(g, key);
    if (!k || k->type != V_STR) return KATALI_ERR_BAD_ARG;
    uint64_t n;
    memcpy(&n, g->map + k->pos, 8);
    *s = reinterpret_cast<const char *>(g->map + k->pos + 8);
    if (len) *len = n;
    return KATALI_OK;
}

int katali_cuda_gguf_array(const KataliGguf *g, const char *key, uint32_t *elem_type, uint64_t *count) {
    if (!g || !key) return KATALI_ERR_BAD_ARG;
    const Kv *k = find_kv(g, key);
    if (!k || k->type != V_ARR) return KATALI_ERR_BAD_ARG;
    if (elem_type) *elem_type = k->elem;
    if (count) *count = k->count;
    return KATALI_OK;
}

int katali_cuda_gguf_array_int(const KataliGguf *g, const char *key, uint64_t i, int64_t *v) {
    if (!g || !key || !v) return KATALI_ERR_BAD_ARG;
    const Kv *k = find_kv(g, key);
    double fv = 0;
    if (!k || k->type != V_ARR || i >= k->count || k->elem == V_STR || k->elem == V_F32 ||
        k->elem == V_F64)
        return KATALI_ERR_BAD_ARG;
    return read_scalar(g, *k, k->elem, k->pos + i * scalar_size(k->elem), v, &fv) ? KATALI_OK
                                                                                  : KATALI_ERR_BAD_ARG;
}

int katali_cuda_gguf_upload(KataliGguf *g, uint64_t i, void *dev) {
    if (!g || !dev || i >= g->t.size()) return KATALI_ERR_BAD_ARG;
    const Tensor &t = g->t[(size_t)i];
    if (!t.nbytes) {
        kq::set_status_message("katali_cuda_gguf_upload: tensor type not sized by this reader");
        return KATALI_ERR_UNSUPPORTED_TYPE;
    }
    // device, own stream and mapped status word (KATALI_ERR_NO_DEVICE without a usable GPU)
    if (const int rs = kq::ensure_runtime()) return rs;
    cudaError_t e = cudaSuccess;
    for (int b = 0; b < 2 && e == cudaSuccess; ++b) {
        if (!g->stage[b]) e = cudaHostAlloc(&g->stage[b], STAGE, cudaHostAllocDefault);
        if (e == cudaSuccess && !g->done[b]) e = cudaEventCreateWithFlags(&g->done[b], cudaEventDisableTiming);
    }
    cudaStream_t st = kq::current_stream();
    const uint8_t *src = g->map + t.abs;
    uint8_t *dst = static_cast<uint8_t *>(dev);
    for (uint64_t off = 0, c = 0; e == cudaSuccess && off < t.nbytes; off += STAGE, ++c) {
        const int b = (int)(c & 1);
        const size_t n = (size_t)(t.nbytes - off < STAGE ? t.nbytes - off : STAGE);
        e = cudaEventSynchronize(g->done[b]);  // the DMA out of this buffer two chunks ago
        if (e != cudaSuccess) break;
        memcpy(g->stage[b], src + off, n);     // page faults pull the file in here
        e = cudaMemcpyAsync(dst + off, g->stage[b], n, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaEventRecord(g->done[b], st);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        kq::set_status_message(cudaGetErrorString(e));
        return e == cudaErrorMemoryAllocation ? KATALI_ERR_OOM : KATALI_ERR_CUDA;
    }
    return KATALI_OK;
}


// A Qwen3-layout dense decoder straight from a model file: metadata (llama.cpp key names under
// the file's general.architecture), tensors by their llama.cpp names (token_embd, output_norm,
// output — the embedding when absent —, blk.N.attn_norm / attn_q / attn_k / attn_v /
// attn_output / attn_q_norm / attn_k_norm / ffn_norm / ffn_gate / ffn_up / ffn_down), every
// tensor uploaded unchanged into one device allocation the decoder then owns.
int katali_cuda_dense_create_from_gguf(KataliGguf *g, uint32_t kv_cap, uint32_t flags,
                                       KataliDense **out) {
    if (!g || !out || !kv_cap) return KATALI_ERR_BAD_ARG;
    *out = nullptr;
    const char *arch = nullptr;
    uint64_t alen = 0;
    if (katali_cuda_gguf_get_str(g, "general.architecture", &arch, &alen) != KATALI_OK)
        return fail(nullptr, "katali_cuda_dense_create_from_gguf: no general.architecture");
    const std::string A(arch, (size_t)alen);
    if (A != "qwen3") {
        kq::set_status_message("katali_cuda_dense_create_from_gguf: architecture is not qwen3");
        return KATALI_ERR_UNSUPPORTED_SHAPE;
    }
    auto meta = [&](const char *key, int64_t def) {
        int64_t v = def;
        if (katali_cuda_gguf_get_int(g, (A + "." + key).c_str(), &v) != KATALI_OK) v = def;
        return v;
    };
    auto metaf = [&](const char *key, double def) {
        double v = def;
        if (katali_cuda_gguf_get_float(g, (A + "." + key).c_str(), &v) != KATALI_OK) v = def;
        return v;
    };
    const int64_t NL = meta("block_count", 0), H = meta("embedding_length", 0),
                  F = meta("feed_forward_length", 0), NH = meta("attention.head_count", 0);
    const int64_t NKV = meta("attention.head_count_kv", NH);
    const int64_t HD = meta("attention.key_length", NH > 0 ? H / NH : 0);
    const int64_t RD = meta("rope.dimension_count", 0);
    if (NL <= 0 || H <= 0 || F <= 0 || NH <= 0 || NKV <= 0 || HD <= 0 || NL > 4096)
        return fail(nullptr, "katali_cuda_dense_create_from_gguf: missing or bad qwen3 dimensions");

    // every tensor: index, with its expected type class (0: fp32 norm, 1: GGUF matrix), dims
    struct Want {
        uint64_t idx;
        uint64_t off;
    };
    std::vector<Want> wants;
    uint64_t total = 0;
    auto take = [&](const std::string &name, bool matrix, uint64_t d0, uint64_t d1, uint64_t *slot,
                    uint32_t *type, bool optional = false) -> int {
        uint64_t i = 0;
        if (katali_cuda_gguf_find(g, name.c_str(), &i) != KATALI_OK) {
            if (optional) {
                *slot = UINT64_MAX;
                return KATALI_OK;
            }
            kq::set_status_message(("katali_cuda_dense_create_from_gguf: missing tensor " + name).c_str());
            return KATALI_ERR_BAD_ARG;
        }
        const Tensor &t = g->t[(size_t)i];
        const bool shape_ok = matrix ? (t.n_dims == 2 && t.dims[0] == d0 && t.dims[1] == d1)
                                     : (t.n_dims == 1 && t.dims[0] == d0 && t.type == 0);
        if (!shape_ok || !t.nbytes) {
            kq::set_status_message(("katali_cuda_dense_create_from_gguf: unexpected shape or type of " + name).c_str());
            return matrix ? KATALI_ERR_UNSUPPORTED_TYPE : KATALI_ERR_BAD_ARG;
        }
        if (type) *type = t.type;
        *slot = wants.size();
        wants.push_back(Want{i, total});
        total += (t.nbytes + 255) & ~(uint64_t)255;
        return KATALI_OK;
    };
    uint64_t emb_i, on_i, lm_i;
    uint32_t emb_t = 0, lm_t = 0;
    uint64_t vocab = 0;
    {
        uint64_t i = 0;
        if (katali_cuda_gguf_find(g, "token_embd.weight", &i) != KATALI_OK || g->t[(size_t)i].n_dims != 2)
            return fail(nullptr, "katali_cuda_dense_create_from_gguf: missing tensor token_embd.weight");
        vocab = g->t[(size_t)i].dims[1];
    }
    int s;
    if ((s = take("token_embd.weight", true, (uint64_t)H, vocab, &emb_i, &emb_t))) return s;
    if ((s = take("output_norm.weight", false, (uint64_t)H, 0, &on_i, nullptr))) return s;
    if ((s = take("output.weight", true, (uint64_t)H, vocab, &lm_i, &lm_t, true))) return s;
    if (lm_i == UINT64_MAX) {  // tied embeddings: the LM head is the embedding matrix
        lm_i = emb_i;
        lm_t = emb_t;
    }
    struct LayerSlots {
        uint64_t an, fn, qn, kn, w[7];
        uint32_t t[7];
    };
    std::vector<LayerSlots> ls((size_t)NL);
    const char *mats[7] = {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"};
    const uint64_t cols[7] = {(uint64_t)H, (uint64_t)H, (uint64_t)H, (uint64_t)(NH * HD),
                              (uint64_t)H, (uint64_t)H, (uint64_t)F};
    const uint64_t rows[7] = {(uint64_t)(NH * HD), (uint64_t)(NKV * HD), (uint64_t)(NKV * HD),
                              (uint64_t)H, (uint64_t)F, (uint64_t)F, (uint64_t)H};
    for (int64_t l = 0; l < NL; ++l) {
        const std::string pfx = "blk." + std::to_string(l) + ".";
        LayerSlots &L = ls[(size_t)l];
        if ((s = take(pfx + "attn_norm.weight", false, (uint64_t)H, 0, &L.an, nullptr))) return s;
        if ((s = take(pfx + "ffn_norm.weight", false, (uint64_t)H, 0, &L.fn, nullptr))) return s;
        if ((s = take(pfx + "attn_q_norm.weight", false, (uint64_t)HD, 0, &L.qn, nullptr, true))) return s;
        if ((s = take(pfx + "attn_k_norm.weight", false, (uint64_t)HD, 0, &L.kn, nullptr, true))) return s;
        for (int j = 0; j < 7; ++j)
            if ((s = take(pfx + mats[j] + ".weight", true, cols[j], rows[j], &L.w[j], &L.t[j]))) return s;
    }
    // device, own stream and mapped status word (KATALI_ERR_NO_DEVICE without a usable GPU)
    if (const int rs = kq::ensure_runtime()) return rs;
    unsigned char *mem = nullptr;
    cudaError_t e = cudaMalloc((void **)&mem, total);
    if (e != cudaSuccess) {
        kq::set_status_message(cudaGetErrorString(e));
        return e == cudaErrorMemoryAllocation ? KATALI_ERR_OOM : KATALI_ERR_CUDA;
    }
    for (const Want &w : wants)
        if ((s = katali_cuda_gguf_upload(g, w.idx, mem + w.off)) != KATALI_OK) {
            cudaFree(mem);
            return s;
        }
    auto ptr = [&](uint64_t slot) -> const void * {
        return slot == UINT64_MAX ? nullptr : mem + wants[(size_t)slot].off;
    };
    std::vector<KataliDenseLayerW> lw((size_t)NL);
    for (int64_t l = 0; l < NL; ++l) {
        const LayerSlots &L = ls[(size_t)l];
        KataliDenseLayerW &w = lw[(size_t)l];
        w.attn_norm = (const float *)ptr(L.an);
        w.ffn_norm = (const float *)ptr(L.fn);
        w.q_norm = (const float *)ptr(L.qn);
        w.k_norm = (const float *)ptr(L.kn);
        const void **m[7] = {&w.wq, &w.wk, &w.wv, &w.wo, &w.gate, &w.up, &w.down};
        uint32_t *t[7] = {&w.wq_type, &w.wk_type, &w.wv_type, &w.wo_type, &w.gate_type, &w.up_type,
                          &w.down_type};
        for (int j = 0; j < 7; ++j) {
            *m[j] = ptr(L.w[j]);
            *t[j] = L.t[j];
        }
    }
    KataliDenseDesc d = {};
    d.n_layers = (uint32_t)NL;
    d.hidden = (uint32_t)H;
    d.ffn = (uint32_t)F;
    d.n_heads = (uint32_t)NH;
    d.n_kv_heads = (uint32_t)NKV;
    d.head_dim = (uint32_t)HD;
    d.vocab = (uint32_t)vocab;
    d.kv_cap = kv_cap;
    d.rope_dim = (uint32_t)(RD > 0 ? RD : 0);
    d.rms_eps = (float)metaf("attention.layer_norm_rms_epsilon", 1e-6);
    d.rope_theta = (float)metaf("rope.freq_base", 1e6);
    d.embed = ptr(emb_i);
    d.embed_type = emb_t;
    d.out_norm = (const float *)ptr(on_i);
    d.lm_head = ptr(lm_i);
    d.lm_head_type = lm_t;
    d.layers = lw.data();
    d.flags = flags;
    s = katali_cuda_dense_create(&d, out);
    if (s != KATALI_OK) {
        cudaFree(mem);
        return s;
    }
    kq::dense_adopt_weights(*out, mem);
    return KATALI_OK;
}


// The hybrid MoE decoder of a qwen35moe file. Non-expert tensors go into one device
// allocation; each layer's stacked experts (expert e's gate rows at e * ffn * row bytes of
// ffn_gate_exps, and so on) either into one allocation per layer (no cache) or, with a cache,
// stay in the mapping and are registered per expert (the stacked tensors page-locked).
int katali_cuda_hybrid_create_from_gguf(KataliGguf *g, uint32_t kv_cap, uint32_t flags,
                                        KataliExpertCache *cache, KataliHybrid **out) {
    if (!g || !out || !kv_cap) return KATALI_ERR_BAD_ARG;
    *out = nullptr;
    const char *arch = nullptr;
    uint64_t alen = 0;
    if (katali_cuda_gguf_get_str(g, "general.architecture", &arch, &alen) != KATALI_OK)
        return fail(nullptr, "katali_cuda_hybrid_create_from_gguf: no general.architecture");
    const std::string A(arch, (size_t)alen);
    if (A != "qwen35moe") {
        kq::set_status_message("katali_cuda_hybrid_create_from_gguf: architecture is not qwen35moe");
        return KATALI_ERR_UNSUPPORTED_SHAPE;
    }
    auto meta = [&](const char *key, int64_t def) {
        int64_t v = def;
        if (katali_cuda_gguf_get_int(g, (A + "." + key).c_str(), &v) != KATALI_OK) v = def;
        return v;
    };
    auto metaf = [&](const char *key, double def) {
        double v = def;
        if (katali_cuda_gguf_get_float(g, (A + "." + key).c_str(), &v) != KATALI_OK) v = def;
        return v;
    };
    const int64_t NL = meta("block_count", 0), H = meta("embedding_length", 0);
    const int64_t NH = meta("attention.head_count", 0), NKV = meta("attention.head_count_kv", NH);
    const int64_t HD = meta("attention.key_length", 0), RD = meta("rope.dimension_count", 0);
    const int64_t E = meta("expert_count", 0), K = meta("expert_used_count", 0);
    const int64_t F = meta("expert_feed_forward_length", 0), CK = meta("ssm.conv_kernel", 0);
    const int64_t DK = meta("ssm.state_size", 0), NK = meta("ssm.group_count", 0);
    const int64_t NV = meta("ssm.time_step_rank", 0), VD = meta("ssm.inner_size", 0);
    const bool norm_topk = meta("expert_weights_norm", 1) != 0;
    if (NL <= 0 || NL > 4096 || H <= 0 || E <= 0 || K <= 0 || K > E || F <= 0)
        return fail(nullptr, "katali_cuda_hybrid_create_from_gguf: missing or bad qwen35moe dimensions");
    const int64_t C = 2 * NK * DK + VD;  // GDN in-projection channels (q, k, v)

    struct Want {
        uint64_t idx, off;
    };
    std::vector<Want> wants;
    uint64_t total = 0;
    const std::string who = "katali_cuda_hybrid_create_from_gguf: ";
    auto find = [&](const std::string &name, uint64_t *i) {
        return katali_cuda_gguf_find(g, name.c_str(), i) == KATALI_OK;
    };
    // a tensor of exact shape (d1 = 0: one dimension; matrix: a GGUF block type), queued for
    // upload into the decoder's allocation
    auto take = [&](const std::string &name, bool matrix, uint64_t d0, uint64_t d1, uint64_t *slot,
                    uint32_t *type, bool optional = false) -> int {
        uint64_t i = 0;
        if (!find(name, &i)) {
            if (optional) {
                *slot = UINT64_MAX;
                return KATALI_OK;
            }
            kq::set_status_message((who + "missing tensor " + name).c_str());
            return KATALI_ERR_BAD_ARG;
        }
        const Tensor &t = g->t[(size_t)i];
        const bool shape_ok = matrix ? (t.n_dims == 2 && t.dims[0] == d0 && t.dims[1] == d1)
                                     : (d1 ? (t.n_dims == 2 && t.dims[0] == d0 && t.dims[1] == d1)
                                           : (t.n_dims == 1 && t.dims[0] == d0)) && t.type == 0;
        if (!shape_ok || !t.nbytes) {
            kq::set_status_message((who + "unexpected shape or type of " + name).c_str());
            return matrix ? KATALI_ERR_UNSUPPORTED_TYPE : KATALI_ERR_BAD_ARG;
        }
        if (type) *type = t.type;
        *slot = wants.size();
        wants.push_back(Want{i, total});
        total += (t.nbytes + 255) & ~(uint64_t)255;
        return KATALI_OK;
    };
    int s;
    uint64_t emb_i, on_i, lm_i, vocab = 0;
    uint32_t emb_t = 0, lm_t = 0;
    {
        uint64_t i = 0;
        if (!find("token_embd.weight", &i) || g->t[(size_t)i].n_dims != 2)
            return fail(nullptr, "katali_cuda_hybrid_create_from_gguf: missing tensor token_embd.weight");
        vocab = g->t[(size_t)i].dims[1];
    }
    if ((s = take("token_embd.weight", true, (uint64_t)H, vocab, &emb_i, &emb_t))) return s;
    if ((s = take("output_norm.weight", false, (uint64_t)H, 0, &on_i, nullptr))) return s;
    if ((s = take("output.weight", true, (uint64_t)H, vocab, &lm_i, &lm_t, true))) return s;
    if (lm_i == UINT64_MAX) {  // tied embeddings
        lm_i = emb_i;
        lm_t = emb_t;
    }
    struct LayerSlots {
        uint32_t kind;
        uint64_t an, fn, rt, w[5], conv, adec, dtb, snorm, qn, kn;
        uint32_t t[5];
        uint64_t exps[3];  // gate, up, down stacked tensors (file indices)
    };
    std::vector<LayerSlots> ls((size_t)NL);
    uint32_t etype[3] = {0, 0, 0};
    for (int64_t l = 0; l < NL; ++l) {
        const std::string pfx = "blk." + std::to_string(l) + ".";
        LayerSlots &L = ls[(size_t)l];
        uint64_t dummy = 0;
        if (find(pfx + "ffn_gate_shexp.weight", &dummy) || find(pfx + "ffn_up_shexp.weight", &dummy)) {
            kq::set_status_message((who + "shared experts (ffn_*_shexp) are not supported").c_str());
            return KATALI_ERR_UNSUPPORTED_SHAPE;
        }
        if ((s = take(pfx + "attn_norm.weight", false, (uint64_t)H, 0, &L.an, nullptr))) return s;
        if ((s = take(pfx + "post_attention_norm.weight", false, (uint64_t)H, 0, &L.fn, nullptr))) return s;
        if ((s = take(pfx + "ffn_gate_inp.weight", false, (uint64_t)H, (uint64_t)E, &L.rt, nullptr))) return s;
        L.kind = find(pfx + "attn_qkv.weight", &dummy) ? KATALI_HYBRID_GDN : KATALI_HYBRID_ATTN;
        if (L.kind == KATALI_HYBRID_GDN) {
            if (C <= 0 || VD <= 0 || NV <= 0 || CK <= 0)
                return fail(nullptr, "katali_cuda_hybrid_create_from_gguf: missing or bad ssm dimensions");
            const char *mats[5] = {"attn_qkv", "attn_gate", "ssm_beta", "ssm_alpha", "ssm_out"};
            const uint64_t cols[5] = {(uint64_t)H, (uint64_t)H, (uint64_t)H, (uint64_t)H, (uint64_t)VD};
            const uint64_t rows[5] = {(uint64_t)C, (uint64_t)VD, (uint64_t)NV, (uint64_t)NV, (uint64_t)H};
            for (int j = 0; j < 5; ++j)
                if ((s = take(pfx + mats[j] + ".weight", true, cols[j], rows[j], &L.w[j], &L.t[j]))) return s;
            if ((s = take(pfx + "ssm_conv1d.weight", false, (uint64_t)CK, (uint64_t)C, &L.conv, nullptr))) return s;
            if ((s = take(pfx + "ssm_a", false, (uint64_t)NV, 0, &L.adec, nullptr))) return s;
            if ((s = take(pfx + "ssm_dt.bias", false, (uint64_t)NV, 0, &L.dtb, nullptr))) return s;
            if ((s = take(pfx + "ssm_norm.weight", false, (uint64_t)DK, 0, &L.snorm, nullptr))) return s;
        } else {
            if (NH <= 0 || NKV <= 0 || HD <= 0)
                return fail(nullptr, "katali_cuda_hybrid_create_from_gguf: missing or bad attention dimensions");
            const char *mats[4] = {"attn_q", "attn_k", "attn_v", "attn_output"};
            const uint64_t cols[4] = {(uint64_t)H, (uint64_t)H, (uint64_t)H, (uint64_t)(NH * HD)};
            const uint64_t rows[4] = {(uint64_t)(2 * NH * HD), (uint64_t)(NKV * HD), (uint64_t)(NKV * HD),
                                      (uint64_t)H};
            for (int j = 0; j < 4; ++j)
                if ((s = take(pfx + mats[j] + ".weight", true, cols[j], rows[j], &L.w[j], &L.t[j]))) return s;
            if ((s = take(pfx + "attn_q_norm.weight", false, (uint64_t)HD, 0, &L.qn, nullptr, true))) return s;
            if ((s = take(pfx + "attn_k_norm.weight", false, (uint64_t)HD, 0, &L.kn, nullptr, true))) return s;
        }
        const char *ex[3] = {"ffn_gate_exps", "ffn_up_exps", "ffn_down_exps"};
        const uint64_t d0[3] = {(uint64_t)H, (uint64_t)H, (uint64_t)F}, d1[3] = {(uint64_t)F, (uint64_t)F, (uint64_t)H};
        for (int j = 0; j < 3; ++j) {
            uint64_t i = 0;
            if (!find(pfx + ex[j] + ".weight", &i)) {
                kq::set_status_message((who + "missing tensor " + pfx + ex[j] + ".weight").c_str());
                return KATALI_ERR_BAD_ARG;
            }
            const Tensor &t = g->t[(size_t)i];
            if (t.n_dims != 3 || t.dims[0] != d0[j] || t.dims[1] != d1[j] || t.dims[2] != (uint64_t)E ||
                !t.nbytes || t.nbytes % (uint64_t)E || (t.nbytes / (uint64_t)E) % 16) {
                kq::set_status_message((who + "unexpected shape or type of " + pfx + ex[j] + ".weight").c_str());
                return KATALI_ERR_UNSUPPORTED_TYPE;
            }
            if (l == 0) etype[j] = t.type;
            else if (t.type != etype[j]) return fail(nullptr, "katali_cuda_hybrid_create_from_gguf: expert types differ between layers");
            L.exps[j] = i;
        }
    }
    if (const int rs = kq::ensure_runtime()) return rs;
    std::vector<void *> allocs;
    std::vector<KataliMoe *> moes;
    std::vector<void *> pinned;
    auto cleanup = [&](int status) {
        for (KataliMoe *m : moes) katali_cuda_moe_destroy(m);
        for (void *a : allocs) cudaFree(a);
        for (void *h : pinned) cudaHostUnregister(h);
        return status;
    };
    auto dev_alloc = [&](uint64_t bytes, unsigned char **p) -> int {
        cudaError_t e = cudaMalloc((void **)p, bytes);
        if (e != cudaSuccess) {
            kq::set_status_message(cudaGetErrorString(e));
            return e == cudaErrorMemoryAllocation ? KATALI_ERR_OOM : KATALI_ERR_CUDA;
        }
        allocs.push_back(*p);
        return KATALI_OK;
    };
    unsigned char *mem = nullptr;
    if ((s = dev_alloc(total, &mem))) return cleanup(s);
    for (const Want &w : wants)
        if ((s = katali_cuda_gguf_upload(g, w.idx, mem + w.off)) != KATALI_OK) return cleanup(s);
    auto ptr = [&](uint64_t slot) -> const void * {
        return slot == UINT64_MAX ? nullptr : mem + wants[(size_t)slot].off;
    };
    // experts: one MoE object per layer, its table on the device copy or left empty for the cache
    std::vector<const void *> table(3 * (size_t)E);
    for (int64_t l = 0; l < NL; ++l) {
        const LayerSlots &L = ls[(size_t)l];
        uint64_t slice[3];
        const uint8_t *host[3];
        for (int j = 0; j < 3; ++j) {
            const Tensor &t = g->t[(size_t)L.exps[j]];
            slice[j] = t.nbytes / (uint64_t)E;
            host[j] = g->map + t.abs;
        }
        if (!cache) {
            unsigned char *ex = nullptr;
            uint64_t off[3], sum = 0;
            for (int j = 0; j < 3; ++j) {
                off[j] = sum;
                sum += (g->t[(size_t)L.exps[j]].nbytes + 255) & ~(uint64_t)255;
            }
            if ((s = dev_alloc(sum, &ex))) return cleanup(s);
            for (int j = 0; j < 3; ++j)
                if ((s = katali_cuda_gguf_upload(g, L.exps[j], ex + off[j])) != KATALI_OK) return cleanup(s);
            for (int64_t e = 0; e < E; ++e)
                for (int j = 0; j < 3; ++j) table[3 * (size_t)e + j] = ex + off[j] + (uint64_t)e * slice[j];
        } else {
            for (int j = 0; j < 3; ++j) {  // page-lock the stacked tensor once (async uploads)
                const uintptr_t pg = 4096, a = (uintptr_t)host[j] & ~(pg - 1);
                const uintptr_t b = ((uintptr_t)host[j] + g->t[(size_t)L.exps[j]].nbytes + pg - 1) & ~(pg - 1);
                if (cudaHostRegister((void *)a, b - a, cudaHostRegisterReadOnly) == cudaSuccess)
                    pinned.push_back((void *)a);
                else
                    cudaGetLastError();
            }
            for (int64_t e = 0; e < E; ++e) {
                s = katali_cuda_expert_register(cache, (uint64_t)l * (uint64_t)E + (uint64_t)e,
                                                host[0] + (uint64_t)e * slice[0], slice[0],
                                                host[1] + (uint64_t)e * slice[1], slice[1],
                                                host[2] + (uint64_t)e * slice[2], slice[2]);
                if (s) return cleanup(s);
            }
            for (auto &p : table) p = nullptr;
        }
        KataliMoeDesc md = {};
        md.n_experts = (uint32_t)E;
        md.hidden = (uint32_t)H;
        md.ffn = (uint32_t)F;
        md.top_k = (uint32_t)K;
        md.gate_type = etype[0];
        md.up_type = etype[1];
        md.down_type = etype[2];
        md.flags = norm_topk ? KATALI_MOE_NORM_TOPK : 0u;
        md.experts = table.data();
        KataliMoe *moe = nullptr;
        if ((s = katali_cuda_moe_create(&md, &moe)) != KATALI_OK) return cleanup(s);
        moes.push_back(moe);
    }
    std::vector<KataliHybridLayerW> lw((size_t)NL);
    for (int64_t l = 0; l < NL; ++l) {
        const LayerSlots &L = ls[(size_t)l];
        KataliHybridLayerW &w = lw[(size_t)l];
        w.kind = L.kind;
        w.attn_norm = (const float *)ptr(L.an);
        w.ffn_norm = (const float *)ptr(L.fn);
        w.router = (const float *)ptr(L.rt);
        w.moe = moes[(size_t)l];
        if (L.kind == KATALI_HYBRID_GDN) {
            w.ssm_qkv = ptr(L.w[0]);
            w.ssm_z = ptr(L.w[1]);
            w.ssm_b = ptr(L.w[2]);
            w.ssm_a = ptr(L.w[3]);
            w.ssm_out = ptr(L.w[4]);
            w.ssm_qkv_type = L.t[0];
            w.ssm_z_type = L.t[1];
            w.ssm_b_type = L.t[2];
            w.ssm_a_type = L.t[3];
            w.ssm_out_type = L.t[4];
            w.ssm_conv = (const float *)ptr(L.conv);
            w.ssm_decay = (const float *)ptr(L.adec);
            w.ssm_dt_bias = (const float *)ptr(L.dtb);
            w.ssm_norm = (const float *)ptr(L.snorm);
        } else {
            w.wq = ptr(L.w[0]);
            w.wk = ptr(L.w[1]);
            w.wv = ptr(L.w[2]);
            w.wo = ptr(L.w[3]);
            w.wq_type = L.t[0];
            w.wk_type = L.t[1];
            w.wv_type = L.t[2];
            w.wo_type = L.t[3];
            w.q_norm = (const float *)ptr(L.qn);
            w.k_norm = (const float *)ptr(L.kn);
        }
    }
    KataliHybridDesc d = {};
    d.n_layers = (uint32_t)NL;
    d.hidden = (uint32_t)H;
    d.vocab = (uint32_t)vocab;
    d.kv_cap = kv_cap;
    d.n_heads = (uint32_t)(NH > 0 ? NH : 0);
    d.n_kv_heads = (uint32_t)(NKV > 0 ? NKV : 0);
    d.head_dim = (uint32_t)(HD > 0 ? HD : 0);
    d.rope_dim = (uint32_t)(RD > 0 ? RD : 0);
    d.rms_eps = (float)metaf("attention.layer_norm_rms_epsilon", 1e-6);
    d.rope_theta = (float)metaf("rope.freq_base", 1e7);
    d.ssm_k_heads = (uint32_t)(NK > 0 ? NK : 0);
    d.ssm_v_heads = (uint32_t)(NV > 0 ? NV : 0);
    d.ssm_head_dim = (uint32_t)(DK > 0 ? DK : 0);
    d.ssm_conv = (uint32_t)(CK > 0 ? CK : 0);
    d.embed = ptr(emb_i);
    d.embed_type = emb_t;
    d.out_norm = (const float *)ptr(on_i);
    d.lm_head = ptr(lm_i);
    d.lm_head_type = lm_t;
    d.layers = lw.data();
    d.flags = flags;
    if ((s = katali_cuda_hybrid_create(&d, out)) != KATALI_OK) return cleanup(s);
    kq::hybrid_adopt(*out, std::move(allocs), std::move(moes), std::move(pinned), cache);
    return KATALI_OK;
}

}  // extern "C"
