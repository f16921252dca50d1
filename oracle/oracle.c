/*
 * oracle.c -- CPU restatement of the reference's fp32 forward pass.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h): the checker for the CUDA path,
 * never part of the product.  Each function cites the reference lines it
 * restates.  All arithmetic is fp32 like the reference's CPUReference; only
 * the RoPE table is computed in double, as RopeTable.swift does.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <errno.h>
#include <float.h>
#include <fcntl.h>
#include <math.h>
#include <omp.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#define MAX_LAYERS 64

/* ------------------------------------------------------------------ GGUF */
/* GGUFValue.swift:83-114: ggml type ids, block sizes and block bytes. */
enum { T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_BF16 = 30 };

typedef struct {
    char* name;
    int ndim;
    int64_t shape[4];
    uint32_t type;
    uint64_t offset;
    const uint8_t* data;
    float* dequant; /* cached fp32 copy, CPUReference.matrix (CPUReference.swift:31-38) */
} tensor_t;

typedef struct {
    char* key;
    uint32_t type;
    const uint8_t* raw; /* position of the value in the mapping */
    uint64_t count;     /* array element count */
    uint32_t elem;      /* array element type */
} kv_t;

struct or_model {
    uint8_t* base;
    size_t size;
    size_t mapped;
    kv_t* kvs;
    int64_t nkv;
    tensor_t* tensors;
    int64_t ntensors;
    or_info info;
    char arch[64];
    int has_ple, has_output, has_dense;
    float embedding_scale, per_layer_scale;
    float* rope[MAX_LAYERS]; /* per layer (shared by head dim and base) */
    int rope_owner[MAX_LAYERS];
    float out_scale[MAX_LAYERS];
    or_vinfo vinfo; /* an mmproj file opened by or_vision_open */
    or_ainfo ainfo; /* an mmproj file opened by or_audio_open */
};

static int set_err(char* err, int errlen, int code, const char* fmt, ...) {
    if (err && errlen > 0) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(err, (size_t)errlen, fmt, ap);
        va_end(ap);
    }
    return code;
}

static int64_t type_block(uint32_t t) { return t == T_Q8_0 ? 32 : 1; }
static int64_t type_bytes(uint32_t t) {
    switch (t) {
    case T_F32: return 4;
    case T_F16: case T_BF16: return 2;
    case T_Q8_0: return 34;
    default: return -1;
    }
}
static int64_t tensor_elems(const tensor_t* t) {
    int64_t n = 1;
    for (int i = 0; i < t->ndim; i++) n *= t->shape[i];
    return n;
}
static int64_t tensor_bytes(const tensor_t* t) { return tensor_elems(t) / type_block(t->type) * type_bytes(t->type); }

typedef struct {
    const uint8_t* base;
    size_t size, pos;
} cursor_t;

static int need(cursor_t* c, size_t n) { return c->pos + n <= c->size; }

/* Skips one metadata value of `type` (GGUFFile.swift:124-176). Returns 0 on success. */
static int skip_value(cursor_t* c, uint32_t type, int depth) {
    static const int64_t fixed[] = {1, 1, 2, 2, 4, 4, 4, 1, -1, -1, 8, 8, 8};
    if (type > 12 || depth > 4) return -1;
    if (type == 8) {
        if (!need(c, 8)) return -1;
        uint64_t n;
        memcpy(&n, c->base + c->pos, 8);
        c->pos += 8;
        if (!need(c, n)) return -1;
        c->pos += n;
        return 0;
    }
    if (type == 9) {
        if (!need(c, 12)) return -1;
        uint32_t et;
        uint64_t n;
        memcpy(&et, c->base + c->pos, 4);
        memcpy(&n, c->base + c->pos + 4, 8);
        c->pos += 12;
        for (uint64_t i = 0; i < n; i++)
            if (skip_value(c, et, depth + 1)) return -1;
        return 0;
    }
    if (!need(c, (size_t)fixed[type])) return -1;
    c->pos += (size_t)fixed[type];
    return 0;
}

static const kv_t* find_kv(const or_model* m, const char* key) {
    for (int64_t i = 0; i < m->nkv; i++)
        if (strcmp(m->kvs[i].key, key) == 0) return &m->kvs[i];
    return NULL;
}

/* GGUFValue.intValue / floatValue (GGUFValue.swift:26-46). */
static int kv_int(const kv_t* kv, int64_t* out) {
    const uint8_t* p = kv->raw;
    switch (kv->type) {
    case 0: *out = *(const uint8_t*)p; return 1;
    case 1: *out = *(const int8_t*)p; return 1;
    case 2: { uint16_t v; memcpy(&v, p, 2); *out = v; return 1; }
    case 3: { int16_t v; memcpy(&v, p, 2); *out = v; return 1; }
    case 4: { uint32_t v; memcpy(&v, p, 4); *out = v; return 1; }
    case 5: { int32_t v; memcpy(&v, p, 4); *out = v; return 1; }
    case 10: { uint64_t v; memcpy(&v, p, 8); *out = (int64_t)v; return 1; }
    case 11: { int64_t v; memcpy(&v, p, 8); *out = v; return 1; }
    default: return 0;
    }
}
static int kv_float(const kv_t* kv, float* out) {
    if (kv->type == 6) { memcpy(out, kv->raw, 4); return 1; }
    if (kv->type == 12) { double d; memcpy(&d, kv->raw, 8); *out = (float)d; return 1; }
    int64_t i;
    if (kv_int(kv, &i)) { *out = (float)i; return 1; }
    return 0;
}

static tensor_t* find_tensor(or_model* m, const char* name) {
    for (int64_t i = 0; i < m->ntensors; i++)
        if (strcmp(m->tensors[i].name, name) == 0) return &m->tensors[i];
    return NULL;
}

static char* read_string(cursor_t* c) {
    if (!need(c, 8)) return NULL;
    uint64_t n;
    memcpy(&n, c->base + c->pos, 8);
    c->pos += 8;
    if (!need(c, n)) return NULL;
    char* s = (char*)malloc(n + 1);
    memcpy(s, c->base + c->pos, n);
    s[n] = 0;
    c->pos += n;
    return s;
}

/* GGUFFile.init (GGUFFile.swift:21-67) over a MAP_SHARED mapping (MappedFile.swift:17-39). */
static int parse_gguf(or_model* m, const char* path, char* err, int errlen) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return set_err(err, errlen, OR_ERR_FILE_NOT_READABLE, "cannot read %s: %s", path, strerror(errno));
    struct stat st;
    if (fstat(fd, &st) != 0) {
        close(fd);
        return set_err(err, errlen, OR_ERR_FILE_NOT_READABLE, "cannot read %s: %s", path, strerror(errno));
    }
    if (st.st_size <= 0) {
        close(fd);
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: file is empty");
    }
    m->size = (size_t)st.st_size;
    long page = sysconf(_SC_PAGESIZE);
    m->mapped = (m->size + (size_t)page - 1) / (size_t)page * (size_t)page;
    void* p = mmap(NULL, m->mapped, PROT_READ, MAP_SHARED, fd, 0);
    close(fd);
    if (p == MAP_FAILED) return set_err(err, errlen, OR_ERR_FILE_NOT_READABLE, "cannot read %s: mmap failed", path);
    m->base = (uint8_t*)p;
    cursor_t c = {m->base, m->size, 0};
    uint32_t magic, version;
    uint64_t ntensors, nkv;
    if (!need(&c, 4)) return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: truncated header at byte 0");
    memcpy(&magic, c.base, 4);
    c.pos = 4;
    if (magic != 0x46554747u) return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: bad magic 0x%x", magic);
    if (!need(&c, 20)) return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: truncated header at byte %zu", c.pos);
    memcpy(&version, c.base + 4, 4);
    if (version != 2 && version != 3)
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: unsupported version %u", version);
    memcpy(&ntensors, c.base + 8, 8);
    memcpy(&nkv, c.base + 16, 8);
    c.pos = 24;
    if (nkv > (1u << 20) || ntensors > (1u << 20))
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: truncated header at byte %zu", c.pos);
    m->kvs = (kv_t*)calloc(nkv ? nkv : 1, sizeof(kv_t));
    for (uint64_t i = 0; i < nkv; i++) {
        char* key = read_string(&c);
        if (!key || !need(&c, 4))
            return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: truncated header at byte %zu", c.pos);
        m->kvs[i].key = key;
        m->nkv = (int64_t)i + 1;
        memcpy(&m->kvs[i].type, c.base + c.pos, 4);
        c.pos += 4;
        uint32_t t = m->kvs[i].type;
        if (t > 12) return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: unknown metadata value type %u", t);
        if (t == 9) {
            if (!need(&c, 12))
                return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: truncated header at byte %zu", c.pos);
            memcpy(&m->kvs[i].elem, c.base + c.pos, 4);
            memcpy(&m->kvs[i].count, c.base + c.pos + 4, 8);
            m->kvs[i].raw = c.base + c.pos + 12;
        } else {
            m->kvs[i].raw = c.base + c.pos;
        }
        if (skip_value(&c, t, 0))
            return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: truncated header at byte %zu", c.pos);
    }
    m->tensors = (tensor_t*)calloc(ntensors ? ntensors : 1, sizeof(tensor_t));
    for (uint64_t i = 0; i < ntensors; i++) {
        tensor_t* t = &m->tensors[i];
        t->name = read_string(&c);
        m->ntensors = (int64_t)i + 1;
        if (!t->name || !need(&c, 4))
            return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: truncated header at byte %zu", c.pos);
        uint32_t nd;
        memcpy(&nd, c.base + c.pos, 4);
        c.pos += 4;
        if (nd > 4) return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: tensor %s has %u dimensions", t->name, nd);
        t->ndim = (int)nd;
        for (uint32_t d = 0; d < nd; d++) {
            if (!need(&c, 8))
                return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: truncated header at byte %zu", c.pos);
            uint64_t s;
            memcpy(&s, c.base + c.pos, 8);
            c.pos += 8;
            t->shape[d] = (int64_t)s;
        }
        if (!need(&c, 12))
            return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: truncated header at byte %zu", c.pos);
        memcpy(&t->type, c.base + c.pos, 4);
        memcpy(&t->offset, c.base + c.pos + 4, 8);
        c.pos += 12;
        if (type_bytes(t->type) < 0)
            return set_err(err, errlen, OR_ERR_UNSUPPORTED_TENSOR_TYPE, "tensor %s uses unsupported storage type %u", t->name, t->type);
    }
    int64_t alignment = 32;
    const kv_t* a = find_kv(m, "general.alignment");
    if (a) {
        int64_t v;
        if (kv_int(a, &v) && v > 0) alignment = v;
    }
    size_t data = (c.pos + (size_t)alignment - 1) / (size_t)alignment * (size_t)alignment;
    for (int64_t i = 0; i < m->ntensors; i++) {
        tensor_t* t = &m->tensors[i];
        if (data + t->offset + (uint64_t)tensor_bytes(t) > m->size)
            return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: tensor %s extends past the end of the file", t->name);
        t->data = m->base + data + t->offset;
    }
    return OR_OK;
}

/* ------------------------------------------------------------------ weights */
static float f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1f, f = h & 0x3ff, bits;
    if (e == 0) {
        if (f == 0) bits = s;
        else { /* subnormal */
            float v = ldexpf((float)f, -24);
            return (h >> 15) ? -v : v;
        }
    } else if (e == 31) bits = s | 0x7f800000u | (f << 13);
    else bits = s | ((e + 112) << 23) | (f << 13);
    float r;
    memcpy(&r, &bits, 4);
    return r;
}

static int64_t tensor_cols(const tensor_t* t) { return t->shape[0]; }
static int64_t tensor_rows(const tensor_t* t) { return tensor_elems(t) / t->shape[0]; }
static int64_t row_bytes(const tensor_t* t) { return tensor_cols(t) / type_block(t->type) * type_bytes(t->type); }

/* WeightTensor.dequantizeRow (Weights.swift:19-43). */
static void dequant_row(const tensor_t* t, int64_t row, float* out) {
    const uint8_t* p = t->data + row * row_bytes(t);
    int64_t n = tensor_cols(t);
    switch (t->type) {
    case T_F32: memcpy(out, p, (size_t)n * 4); break;
    case T_F16:
        for (int64_t i = 0; i < n; i++) { uint16_t h; memcpy(&h, p + 2 * i, 2); out[i] = f16_to_f32(h); }
        break;
    case T_BF16:
        for (int64_t i = 0; i < n; i++) {
            uint16_t h;
            memcpy(&h, p + 2 * i, 2);
            uint32_t b = (uint32_t)h << 16;
            memcpy(&out[i], &b, 4);
        }
        break;
    case T_Q8_0:
        for (int64_t b = 0; b < n / 32; b++) {
            const uint8_t* bp = p + b * 34;
            uint16_t h;
            memcpy(&h, bp, 2);
            float scale = f16_to_f32(h);
            for (int j = 0; j < 32; j++) out[b * 32 + j] = scale * (float)(int8_t)bp[2 + j];
        }
        break;
    }
}

static const float* matrix(or_model* m, tensor_t* t) {
    if (!t->dequant) {
        int64_t rows = tensor_rows(t), cols = tensor_cols(t);
        float* d = (float*)malloc((size_t)(rows * cols) * 4);
#pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < rows; r++) dequant_row(t, r, d + r * cols);
        t->dequant = d;
    }
    (void)m;
    return t->dequant;
}

int or_dequantize_row(or_model* m, const char* name, int64_t row, float* out, int64_t n) {
    tensor_t* t = find_tensor(m, name);
    if (!t) return OR_ERR_MISSING_TENSOR;
    if (row < 0 || row >= tensor_rows(t) || n < tensor_cols(t)) return OR_ERR_INVALID_OPTIONS;
    dequant_row(t, row, out);
    return OR_OK;
}

int or_tensor_shape(or_model* m, const char* name, int64_t* shape, int32_t* ndim) {
    tensor_t* t = find_tensor(m, name);
    if (!t) return OR_ERR_MISSING_TENSOR;
    *ndim = t->ndim;
    for (int i = 0; i < 4; i++) shape[i] = i < t->ndim ? t->shape[i] : 1;
    return OR_OK;
}

/* ModelWeights.init's tensor(name, shape, types) check (Weights.swift:93-98). */
static int check_tensor(or_model* m, const char* name, int64_t s0, int64_t s1, int f32_only, char* err, int errlen,
                        tensor_t** out) {
    tensor_t* t = find_tensor(m, name);
    if (!t) return set_err(err, errlen, OR_ERR_MISSING_TENSOR, "weight file lacks tensor %s", name);
    int want_nd = s1 < 0 ? 1 : 2;
    if (t->ndim != want_nd || t->shape[0] != s0 || (want_nd == 2 && t->shape[1] != s1)) {
        if (want_nd == 1)
            return set_err(err, errlen, OR_ERR_SHAPE_MISMATCH, "tensor %s has shape [%lld], expected [%lld]", name,
                           (long long)t->shape[0], (long long)s0);
        return set_err(err, errlen, OR_ERR_SHAPE_MISMATCH, "tensor %s has shape [%lld, %lld], expected [%lld, %lld]",
                       name, (long long)t->shape[0], (long long)(t->ndim > 1 ? t->shape[1] : 1), (long long)s0,
                       (long long)s1);
    }
    if (f32_only && t->type != T_F32)
        return set_err(err, errlen, OR_ERR_UNSUPPORTED_TENSOR_TYPE, "tensor %s uses unsupported storage type %u", name, t->type);
    if (out) *out = t;
    return OR_OK;
}

/* ModelConfig.init (ModelConfig.swift:54-112), accepting the reference's
 * gemma-embedding2 and the measured gemma-embedding shape. */
static int read_config(or_model* m, char* err, int errlen) {
    const kv_t* a = find_kv(m, "general.architecture");
    if (!a || a->type != 8) return set_err(err, errlen, OR_ERR_UNSUPPORTED_ARCHITECTURE, "unsupported architecture ''");
    uint64_t n;
    memcpy(&n, a->raw, 8);
    if (n >= sizeof(m->arch)) n = sizeof(m->arch) - 1;
    memcpy(m->arch, a->raw + 8, n);
    m->arch[n] = 0;
    if (strcmp(m->arch, "gemma-embedding2") != 0 && strcmp(m->arch, "gemma-embedding") != 0)
        return set_err(err, errlen, OR_ERR_UNSUPPORTED_ARCHITECTURE, "unsupported architecture '%s'", m->arch);
    char key[256];
#define INT_KEY(dst, k)                                                                                 \
    do {                                                                                                \
        snprintf(key, sizeof key, "%s.%s", m->arch, k);                                                 \
        const kv_t* kv_ = find_kv(m, key);                                                              \
        int64_t v_;                                                                                     \
        if (!kv_ || !kv_int(kv_, &v_)) return set_err(err, errlen, OR_ERR_MISSING_METADATA, "weight file lacks metadata key %s", key); \
        dst = (int32_t)v_;                                                                              \
    } while (0)
#define FLOAT_KEY(dst, k)                                                                               \
    do {                                                                                                \
        snprintf(key, sizeof key, "%s.%s", m->arch, k);                                                 \
        const kv_t* kv_ = find_kv(m, key);                                                              \
        if (!kv_ || !kv_float(kv_, &dst)) return set_err(err, errlen, OR_ERR_MISSING_METADATA, "weight file lacks metadata key %s", key); \
    } while (0)
    or_info* I = &m->info;
    INT_KEY(I->layers, "block_count");
    INT_KEY(I->hidden, "embedding_length");
    INT_KEY(I->heads, "attention.head_count");
    if (I->layers <= 0 || I->layers > MAX_LAYERS)
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: %d layers", I->layers);
    snprintf(key, sizeof key, "%s.attention.head_count_kv", m->arch);
    const kv_t* kvh = find_kv(m, key);
    if (!kvh || kvh->type != 9 || (int64_t)kvh->count != I->layers || (kvh->elem != 5 && kvh->elem != 4))
        return set_err(err, errlen, OR_ERR_MISSING_METADATA, "weight file lacks metadata key %s", key);
    snprintf(key, sizeof key, "%s.attention.sliding_window_pattern", m->arch);
    const kv_t* pat = find_kv(m, key);
    if (!pat || pat->type != 9 || pat->elem != 7 || (int64_t)pat->count != I->layers)
        return set_err(err, errlen, OR_ERR_MISSING_METADATA, "weight file lacks metadata key %s", key);
    int32_t hdg, hds, vg, vs;
    INT_KEY(hdg, "attention.key_length");
    INT_KEY(hds, "attention.key_length_swa");
    INT_KEY(vg, "attention.value_length");
    INT_KEY(vs, "attention.value_length_swa");
    if (vg != hdg || vs != hds) return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: key and value head sizes differ");
    float rope_g, rope_s;
    FLOAT_KEY(rope_g, "rope.freq_base");
    snprintf(key, sizeof key, "%s.rope.freq_base_swa", m->arch);
    const kv_t* rs = find_kv(m, key);
    if (!rs || !kv_float(rs, &rope_s)) rope_s = rope_g;
    const kv_t* toks = find_kv(m, "tokenizer.ggml.tokens");
    if (!toks || toks->type != 9 || toks->elem != 8)
        return set_err(err, errlen, OR_ERR_MISSING_METADATA, "weight file lacks metadata key tokenizer.ggml.tokens");
    I->vocab = (int32_t)toks->count;
    INT_KEY(I->out_dim, "embedding_length_out");
    INT_KEY(I->ff, "feed_forward_length");
    INT_KEY(I->per_layer, "embedding_length_per_layer_input");
    INT_KEY(I->sliding_window, "attention.sliding_window");
    FLOAT_KEY(I->eps, "attention.layer_norm_rms_epsilon");
    I->max_tokens = 8192; /* ModelConfig.supportedMaxTokens (ModelConfig.swift:52) */
    for (int i = 0; i < I->layers; i++) {
        int32_t kvn;
        memcpy(&kvn, kvh->raw + 4 * i, 4);
        I->sliding[i] = pat->raw[i] != 0;
        I->kv_heads[i] = kvn;
        I->head_dim[i] = I->sliding[i] ? hds : hdg;
        I->rope_base[i] = I->sliding[i] ? rope_s : rope_g;
    }
    m->embedding_scale = sqrtf((float)I->hidden);
    m->per_layer_scale = 1.0f / sqrtf((float)I->hidden);
    return OR_OK;
#undef INT_KEY
#undef FLOAT_KEY
}

static int check_weights(or_model* m, char* err, int errlen) {
    or_info* I = &m->info;
    int d = I->hidden, ff = I->ff, pl = I->per_layer, rc;
    char name[128];
    if ((rc = check_tensor(m, "token_embd.weight", d, I->vocab, 0, err, errlen, NULL))) return rc;
    m->has_ple = pl > 0;
    if (m->has_ple) {
        if ((rc = check_tensor(m, "per_layer_model_proj.weight", d, (int64_t)pl * I->layers, 0, err, errlen, NULL))) return rc;
        if ((rc = check_tensor(m, "per_layer_proj_norm.weight", pl, -1, 1, err, errlen, NULL))) return rc;
    }
    if ((rc = check_tensor(m, "output_norm.weight", d, -1, 1, err, errlen, NULL))) return rc;
    m->has_output = strcmp(m->arch, "gemma-embedding2") == 0;
    if (m->has_output) {
        if ((rc = check_tensor(m, "output.weight", d, I->out_dim, 0, err, errlen, NULL))) return rc;
        I->dense_head = 0;
    } else {
        tensor_t* t = find_tensor(m, "dense_2.weight");
        if (!t) return set_err(err, errlen, OR_ERR_MISSING_TENSOR, "weight file lacks tensor dense_2.weight");
        I->dense_head = t->ndim == 2 ? (int32_t)t->shape[1] : 0;
        if ((rc = check_tensor(m, "dense_2.weight", d, I->dense_head, 0, err, errlen, NULL))) return rc;
        if ((rc = check_tensor(m, "dense_3.weight", I->dense_head, I->out_dim, 0, err, errlen, NULL))) return rc;
        m->has_dense = 1;
    }
    for (int i = 0; i < I->layers; i++) {
        int hd = I->head_dim[i], qd = I->heads * hd, kvd = I->kv_heads[i] * hd;
#define CHK(suffix, a, b, f32)                                                        \
    snprintf(name, sizeof name, "blk.%d.%s", i, suffix);                              \
    if ((rc = check_tensor(m, name, a, b, f32, err, errlen, NULL))) return rc;
        CHK("attn_norm.weight", d, -1, 1);
        CHK("attn_q.weight", d, qd, 0);
        CHK("attn_k.weight", d, kvd, 0);
        CHK("attn_v.weight", d, kvd, 0);
        CHK("attn_output.weight", qd, d, 0);
        CHK("attn_q_norm.weight", hd, -1, 1);
        CHK("attn_k_norm.weight", hd, -1, 1);
        CHK("post_attention_norm.weight", d, -1, 1);
        CHK("ffn_norm.weight", d, -1, 1);
        CHK("ffn_gate.weight", d, ff, 0);
        CHK("ffn_up.weight", d, ff, 0);
        CHK("ffn_down.weight", ff, d, 0);
        CHK("post_ffw_norm.weight", d, -1, 1);
        m->out_scale[i] = 1.0f;
        if (m->has_ple) {
            CHK("inp_gate.weight", d, pl, 0);
            CHK("proj.weight", pl, d, 0);
            CHK("post_norm.weight", d, -1, 1);
            tensor_t* s;
            snprintf(name, sizeof name, "blk.%d.layer_output_scale.weight", i);
            if ((rc = check_tensor(m, name, 1, -1, 1, err, errlen, &s))) return rc;
            memcpy(&m->out_scale[i], s->data, 4);
        }
#undef CHK
    }
    return OR_OK;
}

void or_close(or_model* m) {
    if (!m) return;
    for (int64_t i = 0; i < m->ntensors; i++) {
        free(m->tensors[i].name);
        free(m->tensors[i].dequant);
    }
    for (int64_t i = 0; i < m->nkv; i++) free(m->kvs[i].key);
    free(m->tensors);
    free(m->kvs);
    for (int i = 0; i < MAX_LAYERS; i++)
        if (m->rope_owner[i]) free(m->rope[i]);
    if (m->base) munmap(m->base, m->mapped);
    free(m);
}

int or_open(const char* path, or_model** out, char* err, int errlen) {
    *out = NULL;
    or_model* m = (or_model*)calloc(1, sizeof(or_model));
    int rc = parse_gguf(m, path, err, errlen);
    if (!rc) rc = read_config(m, err, errlen);
    if (!rc) rc = check_weights(m, err, errlen);
    if (rc) {
        or_close(m);
        return rc;
    }
    /* One table per (head dim, base), as CPUReference.ropeTable caches them (CPUReference.swift:21-28). */
    for (int i = 0; i < m->info.layers; i++) {
        for (int j = 0; j < i; j++)
            if (m->info.head_dim[j] == m->info.head_dim[i] && m->info.rope_base[j] == m->info.rope_base[i]) {
                m->rope[i] = m->rope[j];
                break;
            }
        if (!m->rope[i]) {
            int pairs = m->info.head_dim[i] / 2;
            m->rope[i] = (float*)malloc((size_t)m->info.max_tokens * pairs * 2 * 4);
            or_rope_table(m->info.head_dim[i], m->info.rope_base[i], m->info.max_tokens, m->rope[i]);
            m->rope_owner[i] = 1;
        }
    }
    *out = m;
    return OR_OK;
}

int or_get_info(const or_model* m, or_info* info) {
    *info = m->info;
    return OR_OK;
}

void or_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}
int or_threads(void) { return omp_get_max_threads(); }

/* ------------------------------------------------------------------ math */
/* RopeTable.init (RopeTable.swift:16-31): invFreq = base^(-2i/hd) in double, cos/sin rounded to float. */
void or_rope_table(int32_t head_dim, float base, int32_t positions, float* values) {
    int pairs = head_dim / 2;
    for (int i = 0; i < pairs; i++) {
        double inv = pow((double)base, -2.0 * (double)i / (double)head_dim);
        for (int pos = 0; pos < positions; pos++) {
            double theta = (double)pos * inv;
            values[((size_t)pos * pairs + i) * 2] = (float)cos(theta);
            values[((size_t)pos * pairs + i) * 2 + 1] = (float)sin(theta);
        }
    }
}

typedef float v8 __attribute__((vector_size(32)));

static inline float hsum8(v8 s) { return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7])); }

static inline float dot_tail(const float* a, const float* b, int64_t k0, int64_t k, float s) {
    for (int64_t i = k0; i < k; i++) s += a[i] * b[i];
    return s;
}

/* CPUReference.matmul (CPUReference.swift:63-74): y[M,N] = x[M,K] * w[N,K]^T in fp32.
 * Blocked 4 rows x 2 weight rows; each output is one fixed-order fp32 sum. */
void or_matmul(const float* x, int64_t m, int64_t k, const float* w, int64_t n, float* y) {
    int64_t k8 = k / 8 * 8;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t mb = 0; mb < (m + 3) / 4; mb++) {
        int64_t r0 = mb * 4, rn = m - r0 < 4 ? m - r0 : 4;
        for (int64_t j = 0; j < n; j += 2) {
            int64_t jn = n - j < 2 ? n - j : 2;
            v8 acc[4][2];
            memset(acc, 0, sizeof acc);
            for (int64_t i = 0; i < k8; i += 8) {
                v8 wv[2];
                for (int c = 0; c < jn; c++) memcpy(&wv[c], w + (j + c) * k + i, 32);
                for (int r = 0; r < rn; r++) {
                    v8 xv;
                    memcpy(&xv, x + (r0 + r) * k + i, 32);
                    for (int c = 0; c < jn; c++) acc[r][c] += xv * wv[c];
                }
            }
            for (int r = 0; r < rn; r++)
                for (int c = 0; c < jn; c++)
                    y[(r0 + r) * n + j + c] = dot_tail(x + (r0 + r) * k, w + (j + c) * k, k8, k, hsum8(acc[r][c]));
        }
    }
}

/* CPUReference.rmsNorm (CPUReference.swift:77-90). weight may be NULL. */
void or_rmsnorm(const float* x, int64_t rows, int64_t width, const float* weight, float eps, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        float ss = 0;
        for (int64_t i = 0; i < width; i++) {
            float v = x[r * width + i];
            ss += v * v;
        }
        float inv = 1.0f / sqrtf(ss / (float)width + eps);
        for (int64_t i = 0; i < width; i++) out[r * width + i] = x[r * width + i] * inv * (weight ? weight[i] : 1.0f);
    }
}

/* CPUReference.geluTanh (CPUReference.swift:92-95). */
float or_gelu_tanh(float x) {
    const float c = 0.79788456080286535587989211986876f;
    return 0.5f * x * (1.0f + tanhf(c * x * (1.0f + 0.044715f * x * x)));
}

/* CPUReference.rope (CPUReference.swift:98-113), positions 0..T-1. */
static void rope(float* x, int64_t tokens, int64_t heads, int64_t hd, const float* table) {
    int64_t half = hd / 2;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < tokens; t++)
        for (int64_t h = 0; h < heads; h++) {
            float* o = x + (t * heads + h) * hd;
            for (int64_t i = 0; i < half; i++) {
                float c = table[(t * half + i) * 2], s = table[(t * half + i) * 2 + 1];
                float a = o[i], b = o[i + half];
                o[i] = a * c - b * s;
                o[i + half] = a * s + b * c;
            }
        }
}

/* CPUReference.attention (CPUReference.swift:117-174): bidirectional, GQA, keys with
 * |i - j| > window / 2 masked when window > 0, softmax with expf in fp32.
 * Computed one query row at a time; each row's arithmetic is the reference's. */
void or_attention(const float* q, const float* k, const float* v, int32_t tokens, int32_t heads, int32_t kv_heads,
                  int32_t hd, float scale, int32_t window, float* out) {
    int group = heads / kv_heads;
#pragma omp parallel
    {
        float* s = (float*)malloc((size_t)tokens * 4);
        float* acc = (float*)malloc((size_t)hd * 4);
#pragma omp for schedule(dynamic, 4) collapse(2)
        for (int h = 0; h < heads; h++)
            for (int i = 0; i < tokens; i++) {
                int kh = h / group;
                const float* qi = q + ((int64_t)i * heads + h) * hd;
                float mx = -INFINITY;
                for (int j = 0; j < tokens; j++) {
                    if (window > 0 && abs(i - j) > window / 2) {
                        s[j] = -INFINITY;
                        continue;
                    }
                    const float* kj = k + ((int64_t)j * kv_heads + kh) * hd;
                    v8 a8 = {0};
                    int d = 0;
                    for (; d + 8 <= hd; d += 8) {
                        v8 qa, ka;
                        memcpy(&qa, qi + d, 32);
                        memcpy(&ka, kj + d, 32);
                        a8 += qa * ka;
                    }
                    float dot = dot_tail(qi, kj, d, hd, hsum8(a8));
                    s[j] = dot * scale;
                    if (s[j] > mx) mx = s[j];
                }
                float sum = 0;
                for (int j = 0; j < tokens; j++) {
                    float e = s[j] == -INFINITY ? 0.0f : expf(s[j] - mx);
                    s[j] = e;
                    sum += e;
                }
                float inv = 1.0f / sum;
                for (int d = 0; d < hd; d++) acc[d] = 0;
                for (int j = 0; j < tokens; j++) {
                    float p = s[j] * inv;
                    if (p == 0.0f) continue;
                    const float* vj = v + ((int64_t)j * kv_heads + kh) * hd;
                    for (int d = 0; d < hd; d++) acc[d] += p * vj[d];
                }
                memcpy(out + ((int64_t)i * heads + h) * hd, acc, (size_t)hd * 4);
            }
        free(s);
        free(acc);
    }
}

/* ------------------------------------------------------------------ forward */
static void trace(or_trace_fn fn, void* user, const char* name, const float* data, int64_t n) {
    if (fn) fn(name, data, n, user);
}

static tensor_t* layer_tensor(or_model* m, int l, const char* suffix) {
    char name[128];
    snprintf(name, sizeof name, "blk.%d.%s", l, suffix);
    return find_tensor(m, name);
}

/* CPUReference.forward(rows:trace:) (CPUReference.swift:183-283) over token rows. For the
 * gemma-embedding shape (no per-layer inputs, no output projection) the layer loop is the
 * same without lines 206-210 and 259-270, and the pooled mean of rmsnorm(x, output_norm)
 * goes through dense_2 then dense_3. */
int or_forward(or_model* m, const int32_t* tokens, int32_t T, float* pooled, or_trace_fn tr, void* user) {
    return or_forward_rows(m, tokens, T, NULL, 0, pooled, tr, user);
}

/* A token id below zero, -(r + 1), is row r of `vectors` ([vector_rows][hidden]), entered into
 * the residual stream unscaled (InputRow.vector, CPUReference.swift:191-202). */
int or_forward_rows(or_model* m, const int32_t* tokens, int32_t T, const float* vectors, int64_t vector_rows,
                    float* pooled, or_trace_fn tr, void* user) {
    const or_info* I = &m->info;
    const int64_t d = I->hidden, ff = I->ff, pl = I->per_layer, L = I->layers;
    const float eps = I->eps;
    if (T <= 0 || T > I->max_tokens) return OR_ERR_INVALID_OPTIONS;
    for (int t = 0; t < T; t++)
        if (tokens[t] >= I->vocab || (tokens[t] < 0 && (int64_t)(-(int64_t)tokens[t] - 1) >= vector_rows))
            return OR_ERR_INVALID_OPTIONS;
    char name[64];
    float* x = (float*)malloc((size_t)(T * d) * 4);
    tensor_t* emb = find_tensor(m, "token_embd.weight");
    for (int64_t t = 0; t < T; t++) {
        if (tokens[t] < 0) {
            memcpy(x + t * d, vectors + (-(int64_t)tokens[t] - 1) * d, (size_t)d * 4);
            continue;
        }
        dequant_row(emb, tokens[t], x + t * d);
        for (int64_t i = 0; i < d; i++) x[t * d + i] *= m->embedding_scale;
    }
    trace(tr, user, "inp_scaled", x, T * d);

    float* perLayer = NULL;
    if (m->has_ple) {
        const float* w = matrix(m, find_tensor(m, "per_layer_model_proj.weight"));
        perLayer = (float*)malloc((size_t)(T * pl * L) * 4);
        or_matmul(x, T, d, w, pl * L, perLayer);
        for (int64_t i = 0; i < T * pl * L; i++) perLayer[i] *= m->per_layer_scale;
        or_rmsnorm(perLayer, T * L, pl, matrix(m, find_tensor(m, "per_layer_proj_norm.weight")), eps, perLayer);
        trace(tr, user, "inp_per_layer", perLayer, T * pl * L);
    }

    int64_t maxq = 0, maxkv = 0;
    for (int l = 0; l < L; l++) {
        if (I->heads * I->head_dim[l] > maxq) maxq = I->heads * I->head_dim[l];
        if (I->kv_heads[l] * I->head_dim[l] > maxkv) maxkv = I->kv_heads[l] * I->head_dim[l];
    }
    float* h = (float*)malloc((size_t)(T * d) * 4);
    float* q = (float*)malloc((size_t)(T * maxq) * 4);
    float* k = (float*)malloc((size_t)(T * maxkv) * 4);
    float* v = (float*)malloc((size_t)(T * maxkv) * 4);
    float* attn = (float*)malloc((size_t)(T * maxq) * 4);
    float* o = (float*)malloc((size_t)(T * d) * 4);
    float* gate = (float*)malloc((size_t)(T * ff) * 4);
    float* up = (float*)malloc((size_t)(T * ff) * 4);
    float* g = pl ? (float*)malloc((size_t)(T * pl) * 4) : NULL;

    for (int l = 0; l < L; l++) {
        const int64_t heads = I->heads, kvh = I->kv_heads[l], hd = I->head_dim[l];
        or_rmsnorm(x, T, d, matrix(m, layer_tensor(m, l, "attn_norm.weight")), eps, h);
        snprintf(name, sizeof name, "attn_norm-%d", l); trace(tr, user, name, h, T * d);
        or_matmul(h, T, d, matrix(m, layer_tensor(m, l, "attn_q.weight")), heads * hd, q);
        or_matmul(h, T, d, matrix(m, layer_tensor(m, l, "attn_k.weight")), kvh * hd, k);
        or_matmul(h, T, d, matrix(m, layer_tensor(m, l, "attn_v.weight")), kvh * hd, v);
        snprintf(name, sizeof name, "Qcur-%d", l); trace(tr, user, name, q, T * heads * hd);
        snprintf(name, sizeof name, "Kcur-%d", l); trace(tr, user, name, k, T * kvh * hd);
        snprintf(name, sizeof name, "Vcur-%d", l); trace(tr, user, name, v, T * kvh * hd);
        or_rmsnorm(q, T * heads, hd, matrix(m, layer_tensor(m, l, "attn_q_norm.weight")), eps, q);
        or_rmsnorm(k, T * kvh, hd, matrix(m, layer_tensor(m, l, "attn_k_norm.weight")), eps, k);
        or_rmsnorm(v, T * kvh, hd, NULL, eps, v);
        snprintf(name, sizeof name, "Qcur_normed-%d", l); trace(tr, user, name, q, T * heads * hd);
        snprintf(name, sizeof name, "Kcur_normed-%d", l); trace(tr, user, name, k, T * kvh * hd);
        snprintf(name, sizeof name, "Vcur_normed-%d", l); trace(tr, user, name, v, T * kvh * hd);
        rope(q, T, heads, hd, m->rope[l]);
        rope(k, T, kvh, hd, m->rope[l]);
        snprintf(name, sizeof name, "Qcur_pos-%d", l); trace(tr, user, name, q, T * heads * hd);
        snprintf(name, sizeof name, "Kcur_pos-%d", l); trace(tr, user, name, k, T * kvh * hd);
        or_attention(q, k, v, T, (int32_t)heads, (int32_t)kvh, (int32_t)hd, 1.0f,
                     I->sliding[l] ? I->sliding_window : 0, attn);
        snprintf(name, sizeof name, "kqv_out-%d", l); trace(tr, user, name, attn, T * heads * hd);
        or_matmul(attn, T, heads * hd, matrix(m, layer_tensor(m, l, "attn_output.weight")), d, o);
        or_rmsnorm(o, T, d, matrix(m, layer_tensor(m, l, "post_attention_norm.weight")), eps, o);
        snprintf(name, sizeof name, "attn_post_norm-%d", l); trace(tr, user, name, o, T * d);
        for (int64_t i = 0; i < T * d; i++) x[i] += o[i];
        snprintf(name, sizeof name, "attn_out-%d", l); trace(tr, user, name, x, T * d);

        or_rmsnorm(x, T, d, matrix(m, layer_tensor(m, l, "ffn_norm.weight")), eps, h);
        snprintf(name, sizeof name, "ffn_norm-%d", l); trace(tr, user, name, h, T * d);
        or_matmul(h, T, d, matrix(m, layer_tensor(m, l, "ffn_gate.weight")), ff, gate);
        or_matmul(h, T, d, matrix(m, layer_tensor(m, l, "ffn_up.weight")), ff, up);
        for (int64_t i = 0; i < T * ff; i++) gate[i] = or_gelu_tanh(gate[i]) * up[i];
        snprintf(name, sizeof name, "ffn_geglu-%d", l); trace(tr, user, name, gate, T * ff);
        or_matmul(gate, T, ff, matrix(m, layer_tensor(m, l, "ffn_down.weight")), d, o);
        snprintf(name, sizeof name, "ffn_out-%d", l); trace(tr, user, name, o, T * d);
        or_rmsnorm(o, T, d, matrix(m, layer_tensor(m, l, "post_ffw_norm.weight")), eps, o);
        snprintf(name, sizeof name, "ffn_post_norm-%d", l); trace(tr, user, name, o, T * d);
        for (int64_t i = 0; i < T * d; i++) x[i] += o[i];
        snprintf(name, sizeof name, "pe_in-%d", l); trace(tr, user, name, x, T * d);

        if (m->has_ple) {
            or_matmul(x, T, d, matrix(m, layer_tensor(m, l, "inp_gate.weight")), pl, g);
            for (int64_t t = 0; t < T; t++)
                for (int64_t i = 0; i < pl; i++) {
                    int64_t idx = t * pl + i;
                    g[idx] = or_gelu_tanh(g[idx]) * perLayer[(t * L + l) * pl + i];
                }
            or_matmul(g, T, pl, matrix(m, layer_tensor(m, l, "proj.weight")), d, o);
            or_rmsnorm(o, T, d, matrix(m, layer_tensor(m, l, "post_norm.weight")), eps, o);
            snprintf(name, sizeof name, "per_layer_embd_out-%d", l); trace(tr, user, name, o, T * d);
            for (int64_t i = 0; i < T * d; i++) x[i] = (x[i] + o[i]) * m->out_scale[l];
        }
        snprintf(name, sizeof name, "l_out-%d", l); trace(tr, user, name, x, T * d);
    }

    or_rmsnorm(x, T, d, matrix(m, find_tensor(m, "output_norm.weight")), eps, h);
    trace(tr, user, "result_norm", h, T * d);
    const int64_t od = I->out_dim;
    if (m->has_output) {
        float* proj = (float*)malloc((size_t)(T * od) * 4);
        or_matmul(h, T, d, matrix(m, find_tensor(m, "output.weight")), od, proj);
        trace(tr, user, "result_embd", proj, T * od);
        for (int64_t i = 0; i < od; i++) pooled[i] = 0;
        for (int64_t t = 0; t < T; t++)
            for (int64_t i = 0; i < od; i++) pooled[i] += proj[t * od + i];
        for (int64_t i = 0; i < od; i++) pooled[i] /= (float)T;
        free(proj);
    } else {
        float* mean = (float*)calloc((size_t)d, 4);
        for (int64_t t = 0; t < T; t++)
            for (int64_t i = 0; i < d; i++) mean[i] += h[t * d + i];
        for (int64_t i = 0; i < d; i++) mean[i] /= (float)T;
        trace(tr, user, "result_pooled", mean, d);
        float* mid = (float*)malloc((size_t)I->dense_head * 4);
        or_matmul(mean, 1, d, matrix(m, find_tensor(m, "dense_2.weight")), I->dense_head, mid);
        trace(tr, user, "result_dense_2", mid, I->dense_head);
        or_matmul(mid, 1, I->dense_head, matrix(m, find_tensor(m, "dense_3.weight")), od, pooled);
        trace(tr, user, "result_embd", pooled, od);
        free(mean);
        free(mid);
    }
    free(x); free(h); free(q); free(k); free(v); free(attn); free(o); free(gate); free(up); free(g); free(perLayer);
    return OR_OK;
}

/* ------------------------------------------------------------------ host logic */
/* EmbeddingModel.batches (EmbeddingModel.swift:200-215). batch_size <= 0 means nil.
 * costs is [n][ncost]; ranges receives (start, end) pairs; returns the range count. */
int32_t or_batches(const int64_t* costs, int32_t n, int32_t ncost, int32_t batch_size, const int64_t* budgets,
                   int32_t* ranges) {
    int32_t count = 0, start = 0;
    int64_t totals[16] = {0};
    if (ncost > 16) return -1;
    for (int32_t i = 0; i < n; i++) {
        int full;
        if (batch_size > 0) full = i - start >= batch_size;
        else {
            full = 0;
            for (int c = 0; c < ncost; c++)
                if (totals[c] + costs[(int64_t)i * ncost + c] > budgets[c]) full = 1;
        }
        if (i > start && full) {
            ranges[2 * count] = start;
            ranges[2 * count + 1] = i;
            count++;
            start = i;
            for (int c = 0; c < ncost; c++) totals[c] = 0;
        }
        for (int c = 0; c < ncost; c++) totals[c] += costs[(int64_t)i * ncost + c];
    }
    if (start < n) {
        ranges[2 * count] = start;
        ranges[2 * count + 1] = n;
        count++;
    }
    return count;
}

/* EmbeddingModel.finish (EmbeddingModel.swift:260-267). */
void or_finish(const float* v, int32_t n, int32_t dims, int32_t normalise, float* out) {
    int32_t k = dims < n ? dims : n;
    for (int32_t i = 0; i < k; i++) out[i] = v[i];
    if (normalise) {
        float s = 0;
        for (int32_t i = 0; i < k; i++) s += out[i] * out[i];
        float norm = sqrtf(s);
        if (norm > 0)
            for (int32_t i = 0; i < k; i++) out[i] /= norm;
    }
}

/* SeededRandom.next (Tests/GemmaEmbedTests/KernelTests.swift:14-20). *state holds
 * the generator state (seed + 0x9E3779B97F4A7C15 after init). */
uint64_t or_seeded_next(uint64_t* state) {
    *state += 0x9E3779B97F4A7C15ull;
    uint64_t z = *state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* ------------------------------------------------------------------ vision tower */
static int kv_string_is(const kv_t* kv, const char* want) {
    if (!kv || kv->type != 8) return 0;
    uint64_t n;
    memcpy(&n, kv->raw, 8);
    return n == strlen(want) && memcmp(kv->raw + 8, want, n) == 0;
}

static void kv_string_copy(const kv_t* kv, char* out, size_t cap) {
    out[0] = 0;
    if (!kv || kv->type != 8) return;
    uint64_t n;
    memcpy(&n, kv->raw, 8);
    if (n >= cap) n = cap - 1;
    memcpy(out, kv->raw + 8, n);
    out[n] = 0;
}

/* VisionConfig.init (VisionConfig.swift:42-81). */
static int read_vision_config(or_model* m, char* err, int errlen) {
    char got[64];
    const kv_t* a = find_kv(m, "general.architecture");
    if (!kv_string_is(a, "clip")) {
        kv_string_copy(a, got, sizeof got);
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "image encoder architecture is '%s', expected clip", got);
    }
    const kv_t* pr = find_kv(m, "clip.vision.projector_type");
    if (!kv_string_is(pr, "gemma4v")) {
        kv_string_copy(pr, got, sizeof got);
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "image projector is '%s', expected gemma4v", got);
    }
    or_vinfo* V = &m->vinfo;
#define VINT(dst, k)                                                                                            \
    do {                                                                                                        \
        const kv_t* kv_ = find_kv(m, "clip.vision." k);                                                         \
        int64_t v_;                                                                                             \
        if (!kv_ || !kv_int(kv_, &v_)) return set_err(err, errlen, OR_ERR_MISSING_METADATA, "weight file lacks metadata key clip.vision." k); \
        dst = (int32_t)v_;                                                                                      \
    } while (0)
    const kv_t* e = find_kv(m, "clip.vision.attention.layer_norm_epsilon");
    if (!e || !kv_float(e, &V->eps))
        return set_err(err, errlen, OR_ERR_MISSING_METADATA, "weight file lacks metadata key clip.vision.attention.layer_norm_epsilon");
    VINT(V->hidden, "embedding_length");
    VINT(V->heads, "attention.head_count");
    if (V->heads <= 0 || V->hidden % V->heads)
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "vision width %d does not split into %d heads", V->hidden, V->heads);
    VINT(V->layers, "block_count");
    VINT(V->patch, "patch_size");
    VINT(V->projection_dim, "projection_dim");
    VINT(V->ff, "feed_forward_length");
#undef VINT
    const char* fk[2] = {"clip.vision.image_mean", "clip.vision.image_std"};
    float* fd[2] = {V->mean, V->std};
    for (int i = 0; i < 2; i++) {
        const kv_t* kv = find_kv(m, fk[i]);
        if (!kv || kv->type != 9 || kv->elem != 6 || kv->count != 3)
            return set_err(err, errlen, OR_ERR_MISSING_METADATA, "weight file lacks metadata key %s", fk[i]);
        memcpy(fd[i], kv->raw, 12);
    }
    if (V->layers <= 0 || V->layers > MAX_LAYERS)
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: %d vision layers", V->layers);
    V->head_dim = V->hidden / V->heads;
    V->merge = 3;            /* VisionConfig.swift:29-33: fixed by llama.cpp for gemma4v */
    V->rope_theta = 100.0f;
    return OR_OK;
}

/* VisionWeights.init's shape and type checks (VisionWeights.swift:37-83). */
static int vision_tensor(or_model* m, const char* name, int nd, const int64_t* shape, int types_mask, char* err,
                         int errlen) {
    tensor_t* t = find_tensor(m, name);
    if (!t) return set_err(err, errlen, OR_ERR_MISSING_TENSOR, "weight file lacks tensor %s", name);
    if (shape) {
        int ok = t->ndim == nd;
        for (int i = 0; ok && i < nd; i++) ok = t->shape[i] == shape[i];
        if (!ok) return set_err(err, errlen, OR_ERR_SHAPE_MISMATCH, "tensor %s has an unexpected shape", name);
    }
    int bit = t->type == T_F32 ? 1 : t->type == T_F16 ? 2 : t->type == T_Q8_0 ? 4 : t->type == T_BF16 ? 8 : 0;
    if (!(bit & types_mask))
        return set_err(err, errlen, OR_ERR_UNSUPPORTED_TENSOR_TYPE, "tensor %s uses unsupported storage type %u", name, t->type);
    return OR_OK;
}

static int check_vision_weights(or_model* m, char* err, int errlen) {
    const or_vinfo* V = &m->vinfo;
    const int64_t d = V->hidden, p = V->patch, ff = V->ff, hd = V->head_dim;
    const int ANY = 1 | 2 | 4 | 8, F32 = 1;
    int rc;
    int64_t s4[4] = {p, p, 3, d};
    if ((rc = vision_tensor(m, "v.patch_embd.weight", 4, s4, 1 | 2, err, errlen))) return rc;
    if ((rc = vision_tensor(m, "v.position_embd.weight", 0, NULL, F32, err, errlen))) return rc;
    tensor_t* pos = find_tensor(m, "v.position_embd.weight");
    if (pos->ndim != 3 || pos->shape[0] != d || pos->shape[2] != 2 || pos->shape[1] <= 0)
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "v.position_embd.weight has an unexpected shape");
    m->vinfo.position_count = (int32_t)pos->shape[1];
    int64_t sp[2] = {d, V->projection_dim};
    if ((rc = vision_tensor(m, "mm.input_projection.weight", 2, sp, ANY, err, errlen))) return rc;
    char name[128];
    struct { const char* suffix; int nd; int64_t s0, s1; int types; } L[] = {
        {"ln1.weight", 1, d, 0, F32},          {"attn_q.weight", 2, d, d, ANY},       {"attn_k.weight", 2, d, d, ANY},
        {"attn_v.weight", 2, d, d, ANY},       {"attn_out.weight", 2, d, d, ANY},     {"attn_q_norm.weight", 1, hd, 0, F32},
        {"attn_k_norm.weight", 1, hd, 0, F32}, {"attn_post_norm.weight", 1, d, 0, F32}, {"ln2.weight", 1, d, 0, F32},
        {"ffn_gate.weight", 2, d, ff, ANY},    {"ffn_up.weight", 2, d, ff, ANY},      {"ffn_down.weight", 2, ff, d, ANY},
        {"ffn_post_norm.weight", 1, d, 0, F32},
    };
    for (int l = 0; l < V->layers; l++)
        for (size_t i = 0; i < sizeof L / sizeof L[0]; i++) {
            snprintf(name, sizeof name, "v.blk.%d.%s", l, L[i].suffix);
            int64_t sh[2] = {L[i].s0, L[i].s1};
            if ((rc = vision_tensor(m, name, L[i].nd, sh, L[i].types, err, errlen))) return rc;
        }
    return OR_OK;
}

int or_vision_open(const char* path, or_model** out, char* err, int errlen) {
    *out = NULL;
    or_model* m = (or_model*)calloc(1, sizeof(or_model));
    int rc = parse_gguf(m, path, err, errlen);
    if (!rc) rc = read_vision_config(m, err, errlen);
    if (!rc) rc = check_vision_weights(m, err, errlen);
    if (rc) {
        or_close(m);
        return rc;
    }
    *out = m;
    return OR_OK;
}

int or_vision_get_info(const or_model* v, or_vinfo* info) {
    *info = v->vinfo;
    return OR_OK;
}

/* CPUVisionReference.geluQuick (CPUVisionReference.swift:40-42). */
static float gelu_quick(float x) { return x / (1.0f + expf(-1.702f * x)); }

/* CPUVisionReference.rope2D (CPUVisionReference.swift:46-62): the first half of each head
 * rotates by the patch column, the second by the patch row, each a NeoX rotation of hd / 2
 * dims; `table` holds hd / 4 (cos, sin) pairs per position. */
static void rope_2d(float* x, int64_t tokens, int64_t heads, int64_t hd, const float* table, const int32_t* px,
                    const int32_t* py) {
    const int64_t half = hd / 2, quarter = half / 2;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < tokens; t++)
        for (int axis = 0; axis < 2; axis++) {
            const int64_t offset = axis ? half : 0, pos = axis ? py[t] : px[t];
            for (int64_t h = 0; h < heads; h++) {
                float* o = x + (t * heads + h) * hd + offset;
                for (int64_t i = 0; i < quarter; i++) {
                    const float c = table[(pos * quarter + i) * 2], s = table[(pos * quarter + i) * 2 + 1];
                    const float a = o[i], b = o[i + quarter];
                    o[i] = a * c - b * s;
                    o[i + quarter] = a * s + b * c;
                }
            }
        }
}

/* CPUVisionReference.forward (CPUVisionReference.swift:89-165). */
int or_vision_forward(or_model* m, const float* patches, int32_t gx, int32_t gy, float* out, or_trace_fn tr, void* user) {
    const or_vinfo* V = &m->vinfo;
    const int64_t d = V->hidden, P = (int64_t)gx * gy, heads = V->heads, hd = V->head_dim, ff = V->ff;
    const int64_t area = (int64_t)V->patch * V->patch * 3;
    const float eps = V->eps;
    if (gx <= 0 || gy <= 0 || gx % V->merge || gy % V->merge || gx > V->position_count || gy > V->position_count)
        return OR_ERR_INVALID_OPTIONS;
    char name[64];
    float* x = (float*)malloc((size_t)(P * d) * 4);
    or_matmul(patches, P, area, matrix(m, find_tensor(m, "v.patch_embd.weight")), d, x);
    trace(tr, user, "inp", x, P * d);
    int32_t* px = (int32_t*)malloc((size_t)P * 4);
    int32_t* py = (int32_t*)malloc((size_t)P * 4);
    for (int64_t t = 0; t < P; t++) {
        px[t] = (int32_t)(t % gx);
        py[t] = (int32_t)(t / gx);
    }
    /* v.position_embd.weight as [2 * n][d]: the column table, then the row table. */
    const float* pos = (const float*)find_tensor(m, "v.position_embd.weight")->data;
    for (int64_t t = 0; t < P; t++) {
        for (int64_t i = 0; i < d; i++) x[t * d + i] += pos[(int64_t)px[t] * d + i];
        for (int64_t i = 0; i < d; i++) x[t * d + i] += pos[((int64_t)V->position_count + py[t]) * d + i];
    }
    trace(tr, user, "pos_embd", x, P * d);
    const int32_t npos = gx > gy ? gx : gy;
    float* table = (float*)malloc((size_t)npos * (size_t)(hd / 4) * 2 * 4);
    or_rope_table((int32_t)(hd / 2), V->rope_theta, npos, table);

    float* a = (float*)malloc((size_t)(P * d) * 4);
    float* q = (float*)malloc((size_t)(P * d) * 4);
    float* k = (float*)malloc((size_t)(P * d) * 4);
    float* v = (float*)malloc((size_t)(P * d) * 4);
    float* attn = (float*)malloc((size_t)(P * d) * 4);
    float* o = (float*)malloc((size_t)(P * d) * 4);
    float* gate = (float*)malloc((size_t)(P * ff) * 4);
    float* up = (float*)malloc((size_t)(P * ff) * 4);
#define VW(l, suffix) (snprintf(name, sizeof name, "v.blk.%d." suffix, l), matrix(m, find_tensor(m, name)))
#define TRACE(fmt, l, data, n) (snprintf(name, sizeof name, fmt, l), trace(tr, user, name, data, n))
    for (int l = 0; l < V->layers; l++) {
        or_rmsnorm(x, P, d, VW(l, "ln1.weight"), eps, a);
        TRACE("layer_inp_normed-%d", l, a, P * d);
        or_matmul(a, P, d, VW(l, "attn_q.weight"), d, q);
        or_matmul(a, P, d, VW(l, "attn_k.weight"), d, k);
        or_matmul(a, P, d, VW(l, "attn_v.weight"), d, v);
        TRACE("Vcur-%d", l, v, P * d);
        or_rmsnorm(q, P * heads, hd, VW(l, "attn_q_norm.weight"), eps, q);
        or_rmsnorm(k, P * heads, hd, VW(l, "attn_k_norm.weight"), eps, k);
        TRACE("Qcur-%d", l, q, P * d);
        TRACE("Kcur-%d", l, k, P * d);
        rope_2d(q, P, heads, hd, table, px, py);
        rope_2d(k, P, heads, hd, table, px, py);
        TRACE("Qcur_pos-%d", l, q, P * d);
        TRACE("Kcur_pos-%d", l, k, P * d);
        or_rmsnorm(v, P * heads, hd, NULL, eps, v);
        TRACE("Vcur_normed-%d", l, v, P * d);
        or_attention(q, k, v, (int32_t)P, (int32_t)heads, (int32_t)heads, (int32_t)hd, 1.0f, 0, attn);
        TRACE("kqv_out-%d", l, attn, P * d);
        or_matmul(attn, P, d, VW(l, "attn_out.weight"), d, o);
        TRACE("attn_out-%d", l, o, P * d);
        or_rmsnorm(o, P, d, VW(l, "attn_post_norm.weight"), eps, o);
        TRACE("attn_post_normed-%d", l, o, P * d);
        for (int64_t i = 0; i < P * d; i++) x[i] += o[i];
        TRACE("ffn_inp-%d", l, x, P * d);
        or_rmsnorm(x, P, d, VW(l, "ln2.weight"), eps, a);
        TRACE("ffn_inp_normed-%d", l, a, P * d);
        or_matmul(a, P, d, VW(l, "ffn_gate.weight"), ff, gate);
        or_matmul(a, P, d, VW(l, "ffn_up.weight"), ff, up);
        TRACE("ffn_gate-%d", l, gate, P * ff);
        TRACE("ffn_up-%d", l, up, P * ff);
        for (int64_t i = 0; i < P * ff; i++) gate[i] = gelu_quick(gate[i]) * up[i];
        TRACE("ffn_geglu_quick-%d", l, gate, P * ff);
        or_matmul(gate, P, ff, VW(l, "ffn_down.weight"), d, o);
        TRACE("ffn_out-%d", l, o, P * d);
        or_rmsnorm(o, P, d, VW(l, "ffn_post_norm.weight"), eps, o);
        TRACE("ffn_post_normed-%d", l, o, P * d);
        for (int64_t i = 0; i < P * d; i++) x[i] += o[i];
        TRACE("layer_out-%d", l, x, P * d);
    }
#undef VW
#undef TRACE
    /* CPUVisionReference.pool (CPUVisionReference.swift:66-84). */
    const int64_t mg = V->merge, tx = gx / mg, T = tx * (gy / mg);
    float* pooled = (float*)calloc((size_t)(T * d), 4);
    const float pool_scale = sqrtf((float)d) / (float)(mg * mg);
    for (int64_t oy = 0; oy < gy / mg; oy++)
        for (int64_t ox = 0; ox < tx; ox++) {
            float* dst = pooled + (oy * tx + ox) * d;
            for (int64_t ky = 0; ky < mg; ky++)
                for (int64_t kx = 0; kx < mg; kx++) {
                    const float* src = x + ((oy * mg + ky) * gx + ox * mg + kx) * d;
                    for (int64_t i = 0; i < d; i++) dst[i] += src[i];
                }
            for (int64_t i = 0; i < d; i++) dst[i] *= pool_scale;
        }
    trace(tr, user, "pooled", pooled, T * d);
    or_rmsnorm(pooled, T, d, NULL, eps, pooled);
    or_matmul(pooled, T, d, matrix(m, find_tensor(m, "mm.input_projection.weight")), V->projection_dim, out);
    trace(tr, user, "projected", out, T * V->projection_dim);
    free(x); free(px); free(py); free(table); free(a); free(q); free(k); free(v); free(attn); free(o); free(gate);
    free(up); free(pooled);
    return OR_OK;
}

/* ------------------------------------------------------------------ image preprocessing */
void or_target_size(int32_t width, int32_t height, int32_t alignment, int32_t min_pixels, int32_t max_pixels,
                    int32_t* out_w, int32_t* out_h) {
    const float f = (float)alignment;
#define ROUND_BY(x) ((int32_t)roundf((x) / f) * alignment)
#define CEIL_BY(x) ((int32_t)ceilf((x) / f) * alignment)
#define FLOOR_BY(x) ((int32_t)floorf((x) / f) * alignment)
    int32_t w = ROUND_BY((float)width), h = ROUND_BY((float)height);
    if (w < alignment) w = alignment;
    if (h < alignment) h = alignment;
    if (max_pixels > 0 && (int64_t)w * h > max_pixels) {
        const float beta = sqrtf((float)height * (float)width / (float)max_pixels);
        h = FLOOR_BY((float)height / beta);
        w = FLOOR_BY((float)width / beta);
        if (h < alignment) h = alignment;
        if (w < alignment) w = alignment;
    } else if (min_pixels > 0 && (int64_t)w * h < min_pixels) {
        const float beta = sqrtf((float)min_pixels / ((float)height * (float)width));
        h = CEIL_BY((float)height * beta);
        w = CEIL_BY((float)width * beta);
    }
#undef ROUND_BY
#undef CEIL_BY
#undef FLOOR_BY
    *out_w = w;
    *out_h = h;
}

/* ImageResizer.Kernel (ImageResizer.swift:82-128): Pillow's bicubic taps (a = -0.5) in
 * 22-bit fixed point. */
enum { RS_PRECISION = 22 };

static double bicubic(double x) {
    const double a = -0.5;
    x = fabs(x);
    if (x < 1) return ((a + 2) * x - (a + 3)) * x * x + 1;
    if (x < 2) return (((x - 5) * x + 8) * x - 4) * a;
    return 0;
}

typedef struct {
    int size;
    int* start;
    int* count;
    int32_t* weights;
} rs_kernel;

static rs_kernel rs_make(int in_size, int out_size) {
    rs_kernel k;
    const double support_base = 2.0, scale = (double)in_size / (double)out_size;
    const double filter_scale = scale > 1.0 ? scale : 1.0, support = support_base * filter_scale;
    k.size = (int)ceil(support) * 2 + 1;
    k.start = (int*)calloc((size_t)out_size, sizeof(int));
    k.count = (int*)calloc((size_t)out_size, sizeof(int));
    k.weights = (int32_t*)calloc((size_t)out_size * (size_t)k.size, sizeof(int32_t));
    double* pre = (double*)calloc((size_t)out_size * (size_t)k.size, sizeof(double));
    for (int xx = 0; xx < out_size; xx++) {
        const double center = ((double)xx + 0.5) * scale, ss = 1.0 / filter_scale;
        double ww = 0.0;
        int xmin = (int)(center - support + 0.5);
        if (xmin < 0) xmin = 0;
        int xmax = (int)(center + support + 0.5);
        if (xmax > in_size) xmax = in_size;
        xmax -= xmin;
        for (int x = 0; x < xmax; x++) {
            const double w = bicubic(((double)(x + xmin) - center + 0.5) * ss);
            pre[(size_t)xx * k.size + x] = w;
            ww += w;
        }
        if (ww != 0)
            for (int x = 0; x < xmax; x++) pre[(size_t)xx * k.size + x] /= ww;
        k.start[xx] = xmin;
        k.count[xx] = xmax;
    }
    const double fxp = (double)(1 << RS_PRECISION);
    for (size_t i = 0; i < (size_t)out_size * (size_t)k.size; i++)
        k.weights[i] = (int32_t)(pre[i] * fxp + (pre[i] < 0 ? -0.5 : 0.5));
    free(pre);
    return k;
}

static void rs_free(rs_kernel* k) {
    free(k->start);
    free(k->count);
    free(k->weights);
}

static uint8_t clip8(int32_t v) {
    const int32_t s = v >> RS_PRECISION;
    return (uint8_t)(s < 0 ? 0 : s > 255 ? 255 : s);
}

/* Sums wrap in 32 bits like the reference's &+ and &*. */
static int32_t wrap_mad(int32_t acc, int32_t a, int32_t b) { return (int32_t)((uint32_t)acc + (uint32_t)a * (uint32_t)b); }

/* resizeBicubic (ImageResizer.swift:53-66, 130-176): a horizontal pass, then a vertical pass. */
static uint8_t* resize_bicubic(const uint8_t* in, int w, int h, int tw, int th) {
    const uint8_t* cur = in;
    uint8_t* horiz = NULL;
    int cw = w;
    if (tw != w) {
        rs_kernel k = rs_make(w, tw);
        horiz = (uint8_t*)malloc((size_t)tw * h * 3);
        for (int yy = 0; yy < h; yy++)
            for (int xx = 0; xx < tw; xx++) {
                int32_t s[3] = {1 << (RS_PRECISION - 1), 1 << (RS_PRECISION - 1), 1 << (RS_PRECISION - 1)};
                const uint8_t* p = in + ((size_t)yy * w + k.start[xx]) * 3;
                for (int x = 0; x < k.count[xx]; x++, p += 3) {
                    const int32_t wt = k.weights[(size_t)xx * k.size + x];
                    for (int c = 0; c < 3; c++) s[c] = wrap_mad(s[c], p[c], wt);
                }
                for (int c = 0; c < 3; c++) horiz[((size_t)yy * tw + xx) * 3 + c] = clip8(s[c]);
            }
        rs_free(&k);
        cur = horiz;
        cw = tw;
    }
    uint8_t* out = (uint8_t*)malloc((size_t)cw * th * 3);
    if (th != h) {
        rs_kernel k = rs_make(h, th);
        const size_t row = (size_t)cw * 3;
        int32_t* acc = (int32_t*)malloc(row * 4);
        for (int yy = 0; yy < th; yy++) {
            for (size_t i = 0; i < row; i++) acc[i] = 1 << (RS_PRECISION - 1);
            for (int y = 0; y < k.count[yy]; y++) {
                const int32_t wt = k.weights[(size_t)yy * k.size + y];
                const uint8_t* src = cur + (size_t)(k.start[yy] + y) * row;
                for (size_t i = 0; i < row; i++) acc[i] = wrap_mad(acc[i], src[i], wt);
            }
            for (size_t i = 0; i < row; i++) out[(size_t)yy * row + i] = clip8(acc[i]);
        }
        free(acc);
        rs_free(&k);
    } else {
        memcpy(out, cur, (size_t)cw * th * 3);
    }
    free(horiz);
    return out;
}

void or_fit_image(const uint8_t* in, int32_t w, int32_t h, int32_t tw, int32_t th, uint8_t* out) {
    if (w == tw && h == th) {
        memcpy(out, in, (size_t)w * h * 3);
        return;
    }
    const float sx = (float)tw / (float)w, sy = (float)th / (float)h, scale = sx < sy ? sx : sy;
    int fw = (int)ceilf((float)w * scale), fh = (int)ceilf((float)h * scale);
    if (fw > tw) fw = tw;
    if (fh > th) fh = th;
    uint8_t* fitted = resize_bicubic(in, w, h, fw, fh);
    memset(out, 0, (size_t)tw * th * 3);
    const int ox = (tw - fw) / 2, oy = (th - fh) / 2;
    for (int y = 0; y < fh; y++) memcpy(out + ((size_t)(y + oy) * tw + ox) * 3, fitted + (size_t)y * fw * 3, (size_t)fw * 3);
    free(fitted);
}

/* Round to the nearest fp16 value (ties to even), for normal, subnormal and overflowing inputs. */
float or_round_f16(float x) {
    uint32_t b;
    memcpy(&b, &x, 4);
    const uint32_t sign = b & 0x80000000u, mag = b & 0x7fffffffu;
    if (mag >= 0x7f800000u) return x; /* inf, nan */
    float a;
    memcpy(&a, &mag, 4);
    if (a >= 65520.0f) { /* rounds past the largest finite fp16 */
        uint32_t inf = sign | 0x7f800000u;
        float r;
        memcpy(&r, &inf, 4);
        return r;
    }
    /* Spacing of fp16 values around a: 2^(e - 10) for normals (e >= -14), 2^-24 below. */
    int e;
    frexpf(a, &e); /* a = f * 2^e, f in [0.5, 1) */
    int exp2 = e - 1;
    if (exp2 < -14) exp2 = -14;
    const float ulp = ldexpf(1.0f, exp2 - 10);
    const float q = a / ulp;          /* exact: a scaled by a power of two */
    float r = nearbyintf(q) * ulp;    /* round half to even in the default rounding mode */
    uint32_t rb;
    memcpy(&rb, &r, 4);
    rb |= sign;
    memcpy(&r, &rb, 4);
    return r;
}

void or_patchify(const uint8_t* rgb, int32_t w, int32_t h, int32_t p, const float* mean, const float* std, float* patches) {
    const int32_t gx = w / p, gy = h / p;
    const int64_t area = (int64_t)p * p * 3;
    for (int32_t py = 0; py < gy; py++)
        for (int32_t px = 0; px < gx; px++) {
            const int64_t i = (int64_t)py * gx + px;
            for (int c = 0; c < 3; c++)
                for (int ky = 0; ky < p; ky++)
                    for (int kx = 0; kx < p; kx++) {
                        const uint8_t byte = rgb[(((int64_t)py * p + ky) * w + px * p + kx) * 3 + c];
                        const float f = ((float)byte / 255.0f - mean[c]) / std[c];
                        patches[i * area + (int64_t)c * p * p + ky * p + kx] = or_round_f16(2.0f * f - 1.0f);
                    }
        }
}

/* ------------------------------------------------------------------ gemma4a audio tower */
/* AudioConfig.init (AudioConfig.swift:50-85). */
static int read_audio_config(or_model* m, char* err, int errlen) {
    char got[64];
    const kv_t* a = find_kv(m, "general.architecture");
    if (!kv_string_is(a, "clip")) {
        kv_string_copy(a, got, sizeof got);
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "audio encoder architecture is '%s', expected clip", got);
    }
    const kv_t* has = find_kv(m, "clip.has_audio_encoder");
    if (!has || has->type != 7 || has->raw[0] == 0)
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "the mmproj file has no audio encoder (clip.has_audio_encoder)");
    const kv_t* pr = find_kv(m, "clip.audio.projector_type");
    if (!kv_string_is(pr, "gemma4a")) {
        kv_string_copy(pr, got, sizeof got);
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "audio projector is '%s', expected gemma4a", got);
    }
    or_ainfo* A = &m->ainfo;
#define AINT(dst, k)                                                                                            \
    do {                                                                                                        \
        const kv_t* kv_ = find_kv(m, "clip.audio." k);                                                          \
        int64_t v_;                                                                                             \
        if (!kv_ || !kv_int(kv_, &v_)) return set_err(err, errlen, OR_ERR_MISSING_METADATA, "weight file lacks metadata key clip.audio." k); \
        dst = (int32_t)v_;                                                                                      \
    } while (0)
    AINT(A->hidden, "embedding_length");
    AINT(A->heads, "attention.head_count");
    if (A->heads <= 0 || A->hidden % A->heads)
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "audio width %d does not split into %d heads", A->hidden, A->heads);
    AINT(A->mel_bins, "num_mel_bins");
    if (A->mel_bins % 4)
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "%d mel bins do not survive two stride-2 convolutions evenly", A->mel_bins);
    AINT(A->layers, "block_count");
    AINT(A->ff, "feed_forward_length");
    AINT(A->projection_dim, "projection_dim");
#undef AINT
    tensor_t* o = find_tensor(m, "a.pre_encode.out.weight");
    if (!o || o->ndim != 2 || o->shape[0] != A->hidden)
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "a.pre_encode.out.weight is missing or not [%d, n]", A->hidden);
    A->output_width = (int32_t)o->shape[1];
    if (A->layers <= 0 || A->layers > MAX_LAYERS)
        return set_err(err, errlen, OR_ERR_INVALID_GGUF, "invalid GGUF file: %d audio layers", A->layers);
    A->head_dim = A->hidden / A->heads;
    A->eps = 1e-6f; /* AudioConfig.swift:26-27: fixed, the file's epsilon is ignored */
    A->window = 12;
    A->relative_positions = 13;
    A->softcap = 50.0f;
    A->ff_residual = 0.5f;
    A->dw_kernel = 5;
    A->sub_channels[0] = 128;
    A->sub_channels[1] = 32;
    return OR_OK;
}

/* AudioWeights.init's checks (AudioWeights.swift:67-135). */
static int audio_linear_check(or_model* m, const char* base, int64_t in, int64_t out, char* err, int errlen) {
    char name[128];
    int64_t s[2] = {in, out};
    int rc;
    snprintf(name, sizeof name, "%s.weight", base);
    if ((rc = vision_tensor(m, name, 2, s, 1 | 2 | 4 | 8, err, errlen))) return rc;
    snprintf(name, sizeof name, "%s.bias", base);
    if (find_tensor(m, name) && (rc = vision_tensor(m, name, 1, &s[1], 1, err, errlen))) return rc;
    static const char* bounds[4] = {"input_min", "input_max", "output_min", "output_max"};
    const int64_t one = 1;
    for (int i = 0; i < 4; i++) {
        snprintf(name, sizeof name, "%s.%s", base, bounds[i]);
        if (find_tensor(m, name) && (rc = vision_tensor(m, name, 1, &one, 1, err, errlen))) return rc;
    }
    return OR_OK;
}

static int check_audio_weights(or_model* m, char* err, int errlen) {
    const or_ainfo* A = &m->ainfo;
    const int64_t d = A->hidden, ff = A->ff;
    int rc;
    char name[128];
    int64_t in_c = 1;
    for (int i = 0; i < 2; i++) {
        int64_t s[4] = {3, 3, in_c, A->sub_channels[i]};
        snprintf(name, sizeof name, "a.conv1d.%d.weight", i);
        if ((rc = vision_tensor(m, name, 4, s, 1, err, errlen))) return rc;
        snprintf(name, sizeof name, "a.conv1d.%d.norm.weight", i);
        if ((rc = vision_tensor(m, name, 1, &s[3], 1, err, errlen))) return rc;
        in_c = A->sub_channels[i];
    }
    if ((rc = audio_linear_check(m, "a.input_projection", (int64_t)(A->mel_bins / 4) * A->sub_channels[1], d, err, errlen))) return rc;
    if ((rc = audio_linear_check(m, "a.pre_encode.out", d, A->output_width, err, errlen))) return rc;
    if ((rc = audio_linear_check(m, "mm.a.input_projection", A->output_width, A->projection_dim, err, errlen))) return rc;
    struct { const char* s; int64_t in, out; } lin[] = {
        {"ffn_up", d, ff},   {"ffn_down", ff, d}, {"attn_q", d, d},    {"attn_k", d, d},      {"attn_v", d, d},
        {"attn_out", d, d},  {"attn_k_rel", d, d}, {"conv_pw1", d, 2 * d}, {"conv_pw2", d, d}, {"ffn_up_1", d, ff},
        {"ffn_down_1", ff, d},
    };
    static const char* norms[] = {"ffn_norm", "ffn_post_norm", "attn_pre_norm", "attn_post_norm", "conv_norm",
                                  "norm_conv", "ffn_norm_1", "ffn_post_norm_1", "ln2"};
    for (int l = 0; l < A->layers; l++) {
        for (size_t i = 0; i < sizeof lin / sizeof lin[0]; i++) {
            snprintf(name, sizeof name, "a.blk.%d.%s", l, lin[i].s);
            if ((rc = audio_linear_check(m, name, lin[i].in, lin[i].out, err, errlen))) return rc;
        }
        for (size_t i = 0; i < sizeof norms / sizeof norms[0]; i++) {
            snprintf(name, sizeof name, "a.blk.%d.%s.weight", l, norms[i]);
            if ((rc = vision_tensor(m, name, 1, &d, 1, err, errlen))) return rc;
        }
        const int64_t hd = A->head_dim, dw[2] = {A->dw_kernel, d};
        snprintf(name, sizeof name, "a.blk.%d.per_dim_scale.weight", l);
        if ((rc = vision_tensor(m, name, 1, &hd, 1, err, errlen))) return rc;
        snprintf(name, sizeof name, "a.blk.%d.conv_dw.weight", l);
        if ((rc = vision_tensor(m, name, 2, dw, 1, err, errlen))) return rc;
    }
    return OR_OK;
}

int or_audio_open(const char* path, or_model** out, char* err, int errlen) {
    *out = NULL;
    or_model* m = (or_model*)calloc(1, sizeof(or_model));
    int rc = parse_gguf(m, path, err, errlen);
    if (!rc) rc = read_audio_config(m, err, errlen);
    if (!rc) rc = check_audio_weights(m, err, errlen);
    if (rc) {
        or_close(m);
        return rc;
    }
    *out = m;
    return OR_OK;
}

int or_audio_get_info(const or_model* a, or_ainfo* info) {
    *info = a->ainfo;
    return OR_OK;
}

/* A ClippedLinear's scalar bound, the float range when absent (AudioWeights.swift:89-92). */
static float audio_bound(or_model* m, const char* base, const char* which, float dflt) {
    char name[128];
    snprintf(name, sizeof name, "%s.%s", base, which);
    tensor_t* t = find_tensor(m, name);
    if (!t) return dflt;
    float v;
    memcpy(&v, t->data, 4);
    return v;
}

static void clamp_into(const float* x, int64_t n, float lo, float hi, float* out) {
    for (int64_t i = 0; i < n; i++) out[i] = fminf(fmaxf(x[i], lo), hi);
}

/* CPUAudioReference.linear (CPUAudioReference.swift:51-62): clamp(clamp(x) @ W^T) (+ bias). */
static void audio_linear(or_model* m, const char* base, const float* x, int64_t rows, int64_t in, int64_t out, float* y) {
    char name[128];
    const float in_lo = audio_bound(m, base, "input_min", -FLT_MAX), in_hi = audio_bound(m, base, "input_max", FLT_MAX);
    const float out_lo = audio_bound(m, base, "output_min", -FLT_MAX), out_hi = audio_bound(m, base, "output_max", FLT_MAX);
    float* tmp = NULL;
    if (in_lo != -FLT_MAX || in_hi != FLT_MAX) {
        tmp = (float*)malloc((size_t)(rows * in) * 4);
        clamp_into(x, rows * in, in_lo, in_hi, tmp);
        x = tmp;
    }
    snprintf(name, sizeof name, "%s.weight", base);
    or_matmul(x, rows, in, matrix(m, find_tensor(m, name)), out, y);
    if (out_lo != -FLT_MAX || out_hi != FLT_MAX) clamp_into(y, rows * out, out_lo, out_hi, y);
    snprintf(name, sizeof name, "%s.bias", base);
    tensor_t* b = find_tensor(m, name);
    if (b) {
        const float* bv = (const float*)b->data;
        for (int64_t r = 0; r < rows; r++)
            for (int64_t i = 0; i < out; i++) y[r * out + i] += bv[i];
    }
    free(tmp);
}

/* CPUAudioReference.subsample (CPUAudioReference.swift:67-101): conv kernel 3, stride 2, pad 1
 * over [time][freq][channels] with fp16-rounded inputs, then LayerNorm over the output channels
 * times the norm weight, then ReLU. The weight is [out][channels][3][3]. */
static float* audio_subsample(const float* x, int32_t time, int32_t freq, int32_t channels, const float* w,
                              int32_t out_c, const float* norm, float eps, int32_t* out_time, int32_t* out_freq) {
    const int32_t ot_n = (time - 1) / 2 + 1, of_n = (freq - 1) / 2 + 1;
    const int64_t taps = 9LL * channels;
    float* out = (float*)malloc((size_t)ot_n * of_n * out_c * 4);
#pragma omp parallel for schedule(dynamic, 1)
    for (int32_t ot = 0; ot < ot_n; ot++) {
        float* patch = (float*)malloc((size_t)(of_n * taps) * 4);
        float* col = (float*)malloc((size_t)of_n * out_c * 4);
        for (int32_t of = 0; of < of_n; of++)
            for (int kh = 0; kh < 3; kh++) {
                const int32_t t = 2 * ot + kh - 1;
                for (int kw = 0; kw < 3; kw++) {
                    const int32_t f = 2 * of + kw - 1;
                    const int inside = t >= 0 && t < time && f >= 0 && f < freq;
                    for (int32_t c = 0; c < channels; c++)
                        patch[of * taps + c * 9 + kh * 3 + kw] =
                            inside ? or_round_f16(x[((int64_t)t * freq + f) * channels + c]) : 0.0f;
                }
            }
        for (int32_t of = 0; of < of_n; of++)
            for (int32_t o = 0; o < out_c; o++) {
                const float* a = patch + of * taps;
                const float* b = w + (int64_t)o * taps;
                float s = 0;
                for (int64_t i = 0; i < taps; i++) s += a[i] * b[i];
                col[of * out_c + o] = s;
            }
        for (int32_t of = 0; of < of_n; of++) {
            const float* c = col + of * out_c;
            float mean = 0, var = 0;
            for (int32_t i = 0; i < out_c; i++) mean += c[i];
            mean /= (float)out_c;
            for (int32_t i = 0; i < out_c; i++) var += (c[i] - mean) * (c[i] - mean);
            var /= (float)out_c;
            const float scale = 1.0f / sqrtf(var + eps);
            float* o = out + ((int64_t)ot * of_n + of) * out_c;
            for (int32_t i = 0; i < out_c; i++) o[i] = fmaxf(0.0f, (c[i] - mean) * scale * norm[i]);
        }
        free(patch);
        free(col);
    }
    *out_time = ot_n;
    *out_freq = of_n;
    return out;
}

/* CPUAudioReference.sinusoid (CPUAudioReference.swift:105-115). */
void or_audio_sinusoid(int32_t position, int32_t width, float* out) {
    const int32_t ts = width / 2;
    const float inc = logf(10000.0f) / (float)(ts - 1 > 1 ? ts - 1 : 1);
    for (int32_t i = 0; i < ts; i++) {
        const float scaled = (float)position * expf(-(float)i * inc);
        out[i] = sinf(scaled);
        out[i + ts] = cosf(scaled);
    }
}

/* CPUAudioReference.attention (CPUAudioReference.swift:127-165): query t sees keys t-11..t,
 * scored by content plus the relative key of their distance, capped at softcap*tanh(s/softcap). */
void or_audio_attention(const float* q, const float* k, const float* v, const float* rel, int32_t tokens, int32_t heads,
                        int32_t hd, int32_t window, float softcap, float* out) {
    const int64_t width = (int64_t)heads * hd;
    memset(out, 0, sizeof(float) * (size_t)(tokens * width));
#pragma omp parallel for collapse(2) schedule(static)
    for (int32_t h = 0; h < heads; h++)
        for (int32_t t = 0; t < tokens; t++) {
            float sc[64];
            const int32_t first = t - window + 1 > 0 ? t - window + 1 : 0;
            const float* qr = q + t * width + (int64_t)h * hd;
            float mx = -INFINITY;
            for (int32_t j = first; j <= t; j++) {
                const float* kr = k + j * width + (int64_t)h * hd;
                const float* rr = rel + (int64_t)(t - j) * width + (int64_t)h * hd;
                float s = 0, r = 0;
                for (int32_t i = 0; i < hd; i++) s += qr[i] * kr[i];
                for (int32_t i = 0; i < hd; i++) r += qr[i] * rr[i];
                const float c = softcap * tanhf((s + r) / softcap);
                sc[j - first] = c;
                mx = fmaxf(mx, c);
            }
            float sum = 0;
            for (int32_t j = first; j <= t; j++) {
                sc[j - first] = expf(sc[j - first] - mx);
                sum += sc[j - first];
            }
            float* o = out + t * width + (int64_t)h * hd;
            for (int32_t j = first; j <= t; j++) {
                const float p = sc[j - first] / sum;
                const float* vr = v + j * width + (int64_t)h * hd;
                for (int32_t i = 0; i < hd; i++) o[i] += p * vr[i];
            }
        }
}

/* CPUAudioReference.depthwiseCausal (CPUAudioReference.swift:168-181): w is [width][kernel]. */
void or_audio_depthwise(const float* x, int32_t tokens, int32_t width, const float* w, int32_t kernel, float* out) {
#pragma omp parallel for schedule(static)
    for (int32_t t = 0; t < tokens; t++)
        for (int32_t c = 0; c < width; c++) {
            float s = 0;
            for (int32_t kk = 0; kk < kernel; kk++) {
                const int32_t src = t + kk - (kernel - 1);
                if (src >= 0) s += x[(int64_t)src * width + c] * w[(int64_t)c * kernel + kk];
            }
            out[(int64_t)t * width + c] = s;
        }
}

static float silu(float x) { return x / (1.0f + expf(-x)); }
static float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

/* CPUAudioReference.forward (CPUAudioReference.swift:186-283) over one chunk of `frames` log-mel
 * frames: writes tokens_for_frames(frames) rows of projection_dim values. */
int or_audio_forward(or_model* m, const float* mel, int32_t frames, float* out, or_trace_fn tr, void* user) {
    const or_ainfo* A = &m->ainfo;
    const int64_t d = A->hidden, heads = A->heads, hd = A->head_dim, ff = A->ff;
    const float eps = A->eps;
    if (frames < 1) return OR_ERR_INVALID_OPTIONS;
    char name[96], base[64];
    trace(tr, user, "mel", mel, (int64_t)frames * A->mel_bins);
    int32_t time = frames, freq = A->mel_bins, channels = 1;
    float* act = (float*)malloc((size_t)frames * A->mel_bins * 4);
    memcpy(act, mel, (size_t)frames * A->mel_bins * 4);
    for (int i = 0; i < 2; i++) {
        snprintf(name, sizeof name, "a.conv1d.%d.weight", i);
        const float* w = matrix(m, find_tensor(m, name));
        snprintf(name, sizeof name, "a.conv1d.%d.norm.weight", i);
        const float* nw = matrix(m, find_tensor(m, name));
        int32_t ot, of;
        float* next = audio_subsample(act, time, freq, channels, w, A->sub_channels[i], nw, eps, &ot, &of);
        free(act);
        act = next;
        time = ot;
        freq = of;
        channels = A->sub_channels[i];
        snprintf(name, sizeof name, "subsample-%d", i);
        trace(tr, user, name, act, (int64_t)time * freq * channels);
    }
    const int64_t T = time;
    float* x = (float*)malloc((size_t)(T * d) * 4);
    audio_linear(m, "a.input_projection", act, T, (int64_t)freq * channels, d, x);
    free(act);
    trace(tr, user, "encoder_in", x, T * d);
    float* h = (float*)malloc((size_t)(T * d) * 4);
    float* up = (float*)malloc((size_t)(T * (ff > 2 * d ? ff : 2 * d)) * 4);
    float* down = (float*)malloc((size_t)(T * d) * 4);
    float* q = (float*)malloc((size_t)(T * d) * 4);
    float* k = (float*)malloc((size_t)(T * d) * 4);
    float* v = (float*)malloc((size_t)(T * d) * 4);
    float* attn = (float*)malloc((size_t)(T * d) * 4);
    float* rel = (float*)malloc((size_t)(A->relative_positions * d) * 4);
    float* table = (float*)malloc((size_t)(A->relative_positions * d) * 4);
    for (int32_t p = 0; p < A->relative_positions; p++) or_audio_sinusoid(p, (int32_t)d, table + p * d);
    const float qscale = (1.0f / sqrtf((float)hd)) / logf(2.0f);
    const float kscale = logf(1.0f + expf(1.0f)) / logf(2.0f);
#define AW(l, suffix) (snprintf(name, sizeof name, "a.blk.%d." suffix, l), matrix(m, find_tensor(m, name)))
#define LIN(l, suffix, src, in, outw, dst) (snprintf(base, sizeof base, "a.blk.%d." suffix, l), audio_linear(m, base, src, T, in, outw, dst))
#define TRACE(fmt, l, data, n) (snprintf(name, sizeof name, fmt, l), trace(tr, user, name, data, n))
    for (int l = 0; l < A->layers; l++) {
        /* feed-forward 1, half step */
        or_rmsnorm(x, T, d, AW(l, "ffn_norm.weight"), eps, h);
        TRACE("ffn1_normed-%d", l, h, T * d);
        LIN(l, "ffn_up", h, d, ff, up);
        TRACE("ffn1_up-%d", l, up, T * ff);
        for (int64_t i = 0; i < T * ff; i++) up[i] = silu(up[i]);
        LIN(l, "ffn_down", up, ff, d, down);
        TRACE("ffn1_down-%d", l, down, T * d);
        or_rmsnorm(down, T, d, AW(l, "ffn_post_norm.weight"), eps, down);
        TRACE("ffn1_post_normed-%d", l, down, T * d);
        for (int64_t i = 0; i < T * d; i++) x[i] += A->ff_residual * down[i];
        TRACE("after_ffn1-%d", l, x, T * d);
        /* attention */
        or_rmsnorm(x, T, d, AW(l, "attn_pre_norm.weight"), eps, h);
        TRACE("attn_normed-%d", l, h, T * d);
        LIN(l, "attn_q", h, d, d, q);
        LIN(l, "attn_k", h, d, d, k);
        LIN(l, "attn_v", h, d, d, v);
        TRACE("v-%d", l, v, T * d);
        const float* pds = AW(l, "per_dim_scale.weight");
        for (int64_t t = 0; t < T; t++)
            for (int64_t hh = 0; hh < heads; hh++)
                for (int64_t i = 0; i < hd; i++) q[(t * heads + hh) * hd + i] *= qscale * pds[i];
        for (int64_t i = 0; i < T * d; i++) k[i] *= kscale;
        TRACE("q_scaled-%d", l, q, T * d);
        TRACE("k_scaled-%d", l, k, T * d);
        snprintf(base, sizeof base, "a.blk.%d.attn_k_rel", l);
        audio_linear(m, base, table, A->relative_positions, d, d, rel);
        TRACE("k_rel-%d", l, rel, A->relative_positions * d);
        or_audio_attention(q, k, v, rel, (int32_t)T, (int32_t)heads, (int32_t)hd, A->window, A->softcap, attn);
        TRACE("attn-%d", l, attn, T * d);
        LIN(l, "attn_out", attn, d, d, down);
        TRACE("attn_out-%d", l, down, T * d);
        or_rmsnorm(down, T, d, AW(l, "attn_post_norm.weight"), eps, down);
        for (int64_t i = 0; i < T * d; i++) x[i] += down[i];
        TRACE("after_attn-%d", l, x, T * d);
        /* convolution module */
        or_rmsnorm(x, T, d, AW(l, "conv_norm.weight"), eps, h);
        TRACE("conv_normed-%d", l, h, T * d);
        LIN(l, "conv_pw1", h, d, 2 * d, up);
        TRACE("conv_pw1-%d", l, up, T * 2 * d);
        for (int64_t t = 0; t < T; t++)
            for (int64_t i = 0; i < d; i++) h[t * d + i] = up[t * 2 * d + i] * sigmoidf_(up[t * 2 * d + d + i]);
        TRACE("conv_glu-%d", l, h, T * d);
        or_audio_depthwise(h, (int32_t)T, (int32_t)d, AW(l, "conv_dw.weight"), A->dw_kernel, down);
        TRACE("conv_dw-%d", l, down, T * d);
        or_rmsnorm(down, T, d, AW(l, "norm_conv.weight"), eps, down);
        for (int64_t i = 0; i < T * d; i++) down[i] = silu(down[i]);
        TRACE("conv_silu-%d", l, down, T * d);
        LIN(l, "conv_pw2", down, d, d, attn);
        TRACE("conv_pw2-%d", l, attn, T * d);
        for (int64_t i = 0; i < T * d; i++) x[i] += attn[i];
        TRACE("after_conv-%d", l, x, T * d);
        /* feed-forward 2, half step */
        or_rmsnorm(x, T, d, AW(l, "ffn_norm_1.weight"), eps, h);
        TRACE("ffn2_normed-%d", l, h, T * d);
        LIN(l, "ffn_up_1", h, d, ff, up);
        TRACE("ffn2_up-%d", l, up, T * ff);
        for (int64_t i = 0; i < T * ff; i++) up[i] = silu(up[i]);
        LIN(l, "ffn_down_1", up, ff, d, down);
        TRACE("ffn2_down-%d", l, down, T * d);
        or_rmsnorm(down, T, d, AW(l, "ffn_post_norm_1.weight"), eps, down);
        for (int64_t i = 0; i < T * d; i++) x[i] += A->ff_residual * down[i];
        TRACE("after_ffn2-%d", l, x, T * d);
        or_rmsnorm(x, T, d, AW(l, "ln2.weight"), eps, x);
        TRACE("layer_out-%d", l, x, T * d);
    }
#undef AW
#undef LIN
#undef TRACE
    const int64_t ow = A->output_width;
    float* o = (float*)malloc((size_t)(T * ow) * 4);
    audio_linear(m, "a.pre_encode.out", x, T, d, ow, o);
    trace(tr, user, "out_proj", o, T * ow);
    or_rmsnorm(o, T, ow, NULL, eps, o);
    audio_linear(m, "mm.a.input_projection", o, T, ow, A->projection_dim, out);
    trace(tr, user, "projected", out, T * A->projection_dim);
    free(o);
    free(x);
    free(h);
    free(up);
    free(down);
    free(q);
    free(k);
    free(v);
    free(attn);
    free(rel);
    free(table);
    return OR_OK;
}
