// `.zynfer` model artifacts straight to the device.
//
// The file format is the reference's (src/model/artifact.zig:42-66): an
// 88-byte header, a 116-byte model record, a directory of 120-byte tensor
// entries and a 64-byte-aligned payload, little-endian, with a SHA-256 of the
// whole file (its own field zeroed) in the header. The layout is kept exactly
// so that files written by the reference's converter
// (tools/checkpoint/safetensors_to_zynfer.py) load unchanged. Format version
// 2 adds one dtype tag, 3 = int8: an int8 matrix "X" carries the f32 per-row
// scales of packRowQ8 (ops.zig:145-162) in a companion tensor "X.scale" of
// shape [rows]; nothing else changes, and version-1 files remain valid.
//
// zynfer_cu_artifact_open maps the file read-only (Artifact.loadFile,
// artifact.zig:394-433) and validates it in the reference's order
// (validate, artifact.zig:487-532); errors carry the reference's error names
// (InvalidMagic, UnsupportedVersion, ChecksumMismatch, ...).
// zynfer_cu_load_artifact uploads every tensor of an initialised model by its
// HF name from the mapping (Weights.load, qwen_weights.zig:61-175): f32 and
// bf16 through the regular uploads (int8 models pack them bit-exactly on the
// device), int8 with its scales as they are.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/zynfer_cuda.h"

namespace zc {
// shim.cu: the context's model must exist and have `want`'s architecture
int ctx_check_arch(ZynferCuCtx* c, const ZynferCuModelDesc* want);
int ctx_fail(ZynferCuCtx* c, int code, const char* msg);
}  // namespace zc

namespace {

// ------------------------------------------------------------ SHA-256
// FIPS 180-4, section 6.2: 64 rounds over 512-bit blocks, big-endian words.
const uint32_t kSha256K[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
    0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
    0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
    0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
    0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
    0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
    0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};

struct Sha256 {
    uint32_t h[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                     0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
    uint8_t buf[64];
    size_t fill = 0;
    uint64_t total = 0;

    static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

    void block(const uint8_t* p) {
        uint32_t w[64];
        for (int i = 0; i < 16; ++i)
            w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
        for (int i = 16; i < 64; ++i) {
            const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
            const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
            w[i] = w[i - 16] + s0 + w[i - 7] + s1;
        }
        uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
        for (int i = 0; i < 64; ++i) {
            const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
            const uint32_t ch = (e & f) ^ (~e & g);
            const uint32_t t1 = hh + S1 + ch + kSha256K[i] + w[i];
            const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
            const uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
            const uint32_t t2 = S0 + maj;
            hh = g;
            g = f;
            f = e;
            e = d + t1;
            d = c;
            c = b;
            b = a;
            a = t1 + t2;
        }
        h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
    }

    void update(const uint8_t* p, size_t n) {
        total += n;
        if (fill) {
            const size_t take = n < 64 - fill ? n : 64 - fill;
            memcpy(buf + fill, p, take);
            fill += take;
            p += take;
            n -= take;
            if (fill == 64) {
                block(buf);
                fill = 0;
            }
        }
        while (n >= 64) {
            block(p);
            p += 64;
            n -= 64;
        }
        if (n) {
            memcpy(buf, p, n);
            fill = n;
        }
    }

    void final(uint8_t out[32]) {
        const uint64_t bits = total * 8;
        const uint8_t one = 0x80, zero = 0;
        update(&one, 1);
        while (fill != 56) update(&zero, 1);
        uint8_t len[8];
        for (int i = 0; i < 8; ++i) len[i] = (uint8_t)(bits >> (56 - 8 * i));
        update(len, 8);
        for (int i = 0; i < 8; ++i) {
            out[4 * i] = (uint8_t)(h[i] >> 24);
            out[4 * i + 1] = (uint8_t)(h[i] >> 16);
            out[4 * i + 2] = (uint8_t)(h[i] >> 8);
            out[4 * i + 3] = (uint8_t)h[i];
        }
    }
};

// ------------------------------------------------------ file layout
// artifact.zig:42-66 (Header), 68-122 (Meta), 124-150 (TensorEntry).
constexpr uint32_t kHeaderSize = 88, kMetaSize = 116, kEntrySize = 120;
constexpr uint64_t kPayloadAlign = 64;
constexpr uint64_t kMaxFile = 4ull << 30;  // loadFile's limit (artifact.zig:399)
constexpr size_t kShaOff = 56;              // Header.sha256

// Natural C layout, as Zig's extern structs: 4 padding bytes after
// reserved0 put payload_offset at byte 40.
struct Header {
    char magic[4];
    uint16_t version;
    uint8_t endian, flags;
    uint32_t header_bytes, meta_offset, meta_bytes, dir_offset, dir_bytes, tensor_count, reserved0;
    uint64_t payload_offset, payload_bytes;
    uint8_t sha256[32];
};
struct Meta {
    char model_id[64];
    uint32_t vocab_size, hidden_size, intermediate_size, num_layers, num_attention_heads, num_key_value_heads,
        head_dim, max_position_embeddings, bos_token_id, eos_token_id;
    float rope_theta, rms_norm_eps;
    uint8_t tie_word_embeddings, pad[3];
};
struct Entry {
    char name[64];
    uint32_t tensor_id;
    uint8_t dtype, rank, pad[2];
    uint32_t shape[8];
    uint64_t offset, nbytes;
};
static_assert(sizeof(Header) == kHeaderSize && sizeof(Meta) == kMetaSize && sizeof(Entry) == kEntrySize,
              "layout of format versions 1 and 2");

size_t dtype_size(uint8_t tag) { return tag == ZYNFER_CU_DT_F32 ? 4 : (tag == ZYNFER_CU_DT_I8 ? 1 : 2); }

}  // namespace

struct ZynferCuArtifact {
    std::string err;
    int fd = -1;
    const uint8_t* bytes = nullptr;
    size_t size = 0;
    bool mapped = false;
    std::vector<uint8_t> heap;  // the file when it could not be mapped
    Header h{};
    Meta m{};
    std::vector<Entry> entries;
    std::vector<uint32_t> id_to_index;  // Artifact.buildIdIndex (artifact.zig:305-322)
};

namespace {

int afail(ZynferCuArtifact* a, const std::string& msg) {
    a->err = msg;
    return ZYNFER_CU_INVALID;
}

// validate (artifact.zig:487-532), in its order, plus the version-2 dtype.
int validate(ZynferCuArtifact* a) {
    if (a->size < kHeaderSize) return afail(a, "Truncated: file shorter than the header");
    memcpy(&a->h, a->bytes, kHeaderSize);
    const Header& h = a->h;
    if (memcmp(h.magic, "ZYNF", 4) != 0) return afail(a, "InvalidMagic");
    if (h.version != 1 && h.version != 2) return afail(a, "UnsupportedVersion: " + std::to_string(h.version));
    if (h.endian != 1) return afail(a, "BadEndian");
    if (h.header_bytes != kHeaderSize || h.meta_bytes != kMetaSize || h.meta_offset != kHeaderSize ||
        h.dir_offset != h.meta_offset + h.meta_bytes || (uint64_t)h.dir_bytes != (uint64_t)h.tensor_count * kEntrySize)
        return afail(a, "BadHeader");
    if (h.payload_offset % kPayloadAlign) return afail(a, "BadAlignment: payload offset");
    if (h.payload_offset < (uint64_t)h.dir_offset + h.dir_bytes) return afail(a, "BadHeader: payload overlaps the directory");
    if (a->size < h.payload_offset + h.payload_bytes) return afail(a, "Truncated: payload past the end of the file");
    Sha256 sha;
    static const uint8_t zeros[32] = {0};
    sha.update(a->bytes, kShaOff);
    sha.update(zeros, 32);
    sha.update(a->bytes + kShaOff + 32, a->size - kShaOff - 32);
    uint8_t digest[32];
    sha.final(digest);
    if (memcmp(digest, h.sha256, 32) != 0) return afail(a, "ChecksumMismatch");
    memcpy(&a->m, a->bytes + h.meta_offset, kMetaSize);
    a->entries.resize(h.tensor_count);
    if (h.tensor_count) memcpy(a->entries.data(), a->bytes + h.dir_offset, h.dir_bytes);
    uint32_t max_id = 0;
    for (const Entry& e : a->entries) {
        if (e.rank == 0 || e.rank > 8) return afail(a, "InvalidRank");
        if (e.dtype > ZYNFER_CU_DT_I8 || (e.dtype == ZYNFER_CU_DT_I8 && h.version < 2)) return afail(a, "InvalidDtype");
        if (e.name[0] == 0 || memchr(e.name, 0, sizeof(e.name)) == nullptr) return afail(a, "InvalidName");
        if (e.tensor_id == 0) return afail(a, "InvalidName: tensor id 0");
        if (e.offset + e.nbytes > h.payload_bytes) return afail(a, "Truncated: tensor past the payload");
        if (e.offset % kPayloadAlign) return afail(a, "BadAlignment: tensor offset");
        max_id = e.tensor_id > max_id ? e.tensor_id : max_id;
    }
    if (max_id > 16u * (uint32_t)a->entries.size() + 1024u) return afail(a, "Overflow: sparse tensor ids");
    a->id_to_index.assign((size_t)max_id + 1, UINT32_MAX);
    for (size_t i = 0; i < a->entries.size(); ++i) {
        uint32_t& slot = a->id_to_index[a->entries[i].tensor_id];
        if (slot != UINT32_MAX) return afail(a, "DuplicateTensorId");
        slot = (uint32_t)i;
    }
    return ZYNFER_CU_OK;
}

void fill_info(const ZynferCuArtifact* a, const Entry& e, ZynferCuTensorInfo* out) {
    memset(out, 0, sizeof(*out));
    memcpy(out->name, e.name, sizeof(out->name));
    out->tensor_id = e.tensor_id;
    out->dtype = e.dtype;
    out->rank = e.rank;
    for (int i = 0; i < 8; ++i) out->shape[i] = e.shape[i];
    out->nbytes = e.nbytes;
    out->data = a->bytes + a->h.payload_offset + e.offset;
}

const Entry* find_name(const ZynferCuArtifact* a, const char* name) {
    for (const Entry& e : a->entries)
        if (strncmp(e.name, name, sizeof(e.name)) == 0) return &e;
    return nullptr;
}

uint64_t elems(const Entry& e) {
    uint64_t n = 1;
    for (int i = 0; i < e.rank; ++i) n *= e.shape[i];
    return n;
}

}  // namespace

extern "C" {

int zynfer_cu_artifact_open(const char* path, ZynferCuArtifact** out) {
    if (!out) return ZYNFER_CU_INVALID;
    ZynferCuArtifact* a = new ZynferCuArtifact();
    *out = a;
    if (!path) return afail(a, "InvalidName: no path");
    a->fd = open(path, O_RDONLY);
    if (a->fd < 0) return afail(a, std::string("FileNotFound: ") + path);
    struct stat st;
    if (fstat(a->fd, &st) != 0) return afail(a, "FileNotFound: stat failed");
    if ((uint64_t)st.st_size > kMaxFile) return afail(a, "Overflow: larger than 4 GiB");
    if (st.st_size == 0) return afail(a, "Truncated: empty file");
    a->size = (size_t)st.st_size;
    void* p = mmap(nullptr, a->size, PROT_READ, MAP_PRIVATE, a->fd, 0);
    if (p != MAP_FAILED) {
        a->bytes = static_cast<const uint8_t*>(p);
        a->mapped = true;
    } else {  // the heap copy loadFile falls back to
        a->heap.resize(a->size);
        size_t off = 0;
        while (off < a->size) {
            const ssize_t r = pread(a->fd, a->heap.data() + off, a->size - off, (off_t)off);
            if (r <= 0) break;
            off += (size_t)r;
        }
        if (off != a->size) return afail(a, "Truncated: short read");
        a->bytes = a->heap.data();
    }
    return validate(a);
}

void zynfer_cu_artifact_close(ZynferCuArtifact* a) {
    if (!a) return;
    if (a->mapped) munmap(const_cast<uint8_t*>(a->bytes), a->size);
    if (a->fd >= 0) close(a->fd);
    delete a;
}

const char* zynfer_cu_artifact_error(const ZynferCuArtifact* a) { return a ? a->err.c_str() : "null artifact"; }

int zynfer_cu_artifact_meta(const ZynferCuArtifact* a, ZynferCuArtifactMeta* out) {
    if (!a || !out || a->entries.size() != a->h.tensor_count || !a->bytes) return ZYNFER_CU_INVALID;
    memset(out, 0, sizeof(*out));
    memcpy(out->model_id, a->m.model_id, sizeof(out->model_id));
    out->model_id[sizeof(out->model_id) - 1] = 0;
    out->format_version = a->h.version;
    out->vocab = a->m.vocab_size;
    out->hidden = a->m.hidden_size;
    out->inter = a->m.intermediate_size;
    out->layers = a->m.num_layers;
    out->n_q = a->m.num_attention_heads;
    out->n_kv = a->m.num_key_value_heads;
    out->head_dim = a->m.head_dim;
    out->max_pos = a->m.max_position_embeddings;
    out->bos = a->m.bos_token_id;
    out->eos = a->m.eos_token_id;
    out->rope_theta = a->m.rope_theta;
    out->rms_norm_eps = a->m.rms_norm_eps;
    out->tie_word_embeddings = a->m.tie_word_embeddings;
    out->tensor_count = a->h.tensor_count;
    out->file_bytes = a->size;
    return ZYNFER_CU_OK;
}

int zynfer_cu_artifact_tensor(const ZynferCuArtifact* a, uint32_t index, ZynferCuTensorInfo* out) {
    if (!a || !out || index >= a->entries.size()) return ZYNFER_CU_INVALID;
    fill_info(a, a->entries[index], out);
    return ZYNFER_CU_OK;
}

int zynfer_cu_artifact_find_id(const ZynferCuArtifact* a, uint32_t tensor_id, ZynferCuTensorInfo* out) {
    if (!a || !out) return ZYNFER_CU_INVALID;
    if (tensor_id >= a->id_to_index.size() || a->id_to_index[tensor_id] == UINT32_MAX) return ZYNFER_CU_INVALID;
    fill_info(a, a->entries[a->id_to_index[tensor_id]], out);
    return ZYNFER_CU_OK;
}

int zynfer_cu_artifact_find_name(const ZynferCuArtifact* a, const char* name, ZynferCuTensorInfo* out) {
    if (!a || !name || !out) return ZYNFER_CU_INVALID;
    const Entry* e = find_name(a, name);
    if (!e) return ZYNFER_CU_INVALID;
    fill_info(a, *e, out);
    return ZYNFER_CU_OK;
}

int zynfer_cu_model_desc_from_artifact(const ZynferCuArtifact* a, ZynferCuModelDesc* desc) {
    if (!a || !desc || !a->bytes || a->entries.size() != a->h.tensor_count) return ZYNFER_CU_INVALID;
    desc->vocab = a->m.vocab_size;
    desc->hidden = a->m.hidden_size;
    desc->inter = a->m.intermediate_size;
    desc->layers = a->m.num_layers;
    desc->n_q = a->m.num_attention_heads;
    desc->n_kv = a->m.num_key_value_heads;
    desc->head_dim = a->m.head_dim;
    desc->max_pos = a->m.max_position_embeddings;
    desc->eps = a->m.rms_norm_eps;
    desc->theta = a->m.rope_theta;
    return ZYNFER_CU_OK;
}

int zynfer_cu_load_artifact(ZynferCuCtx* ctx, const ZynferCuArtifact* a) {
    if (!ctx || !a || !a->bytes || a->entries.size() != a->h.tensor_count) return ZYNFER_CU_INVALID;
    // the model's architecture must be the artifact's (Weights.load, qwen_weights.zig:61-65)
    ZynferCuModelDesc want{};
    zynfer_cu_model_desc_from_artifact(a, &want);
    int rc = zc::ctx_check_arch(ctx, &want);
    if (rc) return rc;
    if (!a->m.tie_word_embeddings) return zc::ctx_fail(ctx, ZYNFER_CU_UNSUPPORTED, "untied LM head: this backend ties it to the embedding");
    std::vector<std::string> names = {"model.embed_tokens.weight", "model.norm.weight"};
    static const char* per_layer[11] = {"input_layernorm.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
                                        "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                                        "self_attn.o_proj.weight", "post_attention_layernorm.weight",
                                        "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"};
    char buf[96];
    for (uint32_t l = 0; l < a->m.num_layers; ++l)
        for (const char* n : per_layer) {
            snprintf(buf, sizeof(buf), "model.layers.%u.%s", l, n);
            names.emplace_back(buf);
        }
    for (const std::string& name : names) {
        const Entry* e = find_name(a, name.c_str());
        if (!e) return zc::ctx_fail(ctx, ZYNFER_CU_INVALID, ("TensorNotFound: " + name).c_str());
        const uint64_t n = elems(*e);
        if (e->nbytes != n * dtype_size(e->dtype))
            return zc::ctx_fail(ctx, ZYNFER_CU_INVALID, ("ShapeMismatch: byte count of " + name).c_str());
        const uint64_t rows = e->shape[0], cols = e->rank >= 2 ? n / e->shape[0] : 1;
        const void* data = a->bytes + a->h.payload_offset + e->offset;
        switch (e->dtype) {
            case ZYNFER_CU_DT_F32:
                rc = zynfer_cu_upload_f32(ctx, name.c_str(), static_cast<const float*>(data), rows, cols);
                break;
            case ZYNFER_CU_DT_BF16:
                rc = zynfer_cu_upload_bf16(ctx, name.c_str(), static_cast<const uint16_t*>(data), rows, cols);
                break;
            case ZYNFER_CU_DT_I8: {
                const std::string sname = name + ".scale";
                const Entry* s = find_name(a, sname.c_str());
                if (!s || s->dtype != ZYNFER_CU_DT_F32 || s->rank != 1 || s->shape[0] != rows || s->nbytes != rows * 4)
                    return zc::ctx_fail(ctx, ZYNFER_CU_INVALID, ("TensorNotFound: f32 [rows] " + sname).c_str());
                rc = zynfer_cu_upload_q8(ctx, name.c_str(), static_cast<const int8_t*>(data),
                                         reinterpret_cast<const float*>(a->bytes + a->h.payload_offset + s->offset), rows,
                                         cols);
                break;
            }
            default:  // f16: decodeWeights rejects it (qwen_weights.zig:230)
                return zc::ctx_fail(ctx, ZYNFER_CU_INVALID, ("InvalidDtype: f16 " + name).c_str());
        }
        if (rc) return rc;
    }
    return ZYNFER_CU_OK;
}

}  // extern "C"
