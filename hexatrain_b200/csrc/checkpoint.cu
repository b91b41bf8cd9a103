// checkpoint.cu -- NPRTCKPTV2/V3 checkpoint codec for the LM training state
// and bit-exact resume on top of the device state.
//
// Byte layout (qnn/qnn_transformer_training.cpp:5164-5252, writer;
// :5390-5522, reader):
//   "NPRTCKPTV2\n" (or V3 at the 1024-entry byte-BPE vocabulary, V1 =
//   parameters only, read-only here)
//   u32 vocab, tokens, dimension, ffn, layers, heads, seed, step (big endian)
//   V3 only: u32 kind length, kind ("byte_bpe"), u32 hash length (71),
//            hash ("sha256:" + 64 hex)
//   three registries -- parameters, Adam first moments, Adam second moments
//   -- each: u32 entry count, then per entry u32 name length, name,
//   u64 element count (big endian), the float32 values as stored in memory
//   (little endian).  Nothing may follow.
// Registry order and names are tiny_lm::parameterRegistry
// (tiny_language_model_cpu.cpp:63): token_embedding, layer_%03d.{norm1_gamma,
// norm1_beta, wq, wk, wv, wo, norm2_gamma, norm2_beta, ffn_w1, ffn_w2},
// output_projection -- the order of the flat parameter buffer here.  A
// learned-position model (HX_LM_LEARNED_POSITION, not in the reference)
// carries one more entry, position_embedding, right after token_embedding.
//
// Writer rules kept from the reference: step 0 and non-finite state are
// refused; the tokenizer block is present exactly at vocabulary 1024 (kind
// "byte_bpe", hash of 71 characters starting "sha256:"); files are written
// to "<path>.tmp" and renamed over the destination.  Reader rules: 64 MiB
// size cap, magic, configuration and seed identity, tokenizer identity,
// step in [1, 999999], registry count, order, names (1..256 bytes) and
// element counts, Adam registries for V2/V3, no trailing bytes; non-finite
// values are reported (finite = 0) rather than rejected, as the reference's
// generation loader does.  Error strings are the reference's codes.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "plans.cuh"

namespace hx {
namespace {

constexpr uint64_t kNprtMaxBytes = 64ull * 1024 * 1024;
constexpr uint32_t kBpeVocabulary = 1024;
constexpr uint64_t kFnvOffset = 14695981039346656037ull;
constexpr uint64_t kFnvPrime = 1099511628211ull;

struct Entry {
    std::string name;
    uint64_t count;
};

std::vector<Entry> registry(const hx_lm_config& c) {
    const uint64_t V = c.vocab, T = c.tokens, D = c.dim, F = c.ffn;
    std::vector<Entry> r;
    r.push_back({"token_embedding", V * D});
    if (c.flags & HX_LM_LEARNED_POSITION) r.push_back({"position_embedding", T * D});
    for (uint32_t l = 0; l < c.layers; ++l) {
        char pre[32];
        std::snprintf(pre, sizeof pre, "layer_%03u.", l);
        const std::string p(pre);
        r.push_back({p + "norm1_gamma", D});
        r.push_back({p + "norm1_beta", D});
        r.push_back({p + "wq", D * D});
        r.push_back({p + "wk", D * D});
        r.push_back({p + "wv", D * D});
        r.push_back({p + "wo", D * D});
        r.push_back({p + "norm2_gamma", D});
        r.push_back({p + "norm2_beta", D});
        r.push_back({p + "ffn_w1", D * F});
        r.push_back({p + "ffn_w2", F * D});
    }
    r.push_back({"output_projection", D * V});
    return r;
}

uint64_t total(const std::vector<Entry>& r) {
    uint64_t n = 0;
    for (const auto& e : r) n += e.count;
    return n;
}

bool all_finite(const float* p, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i)
        if (!std::isfinite(p[i])) return false;
    return true;
}

bool tokenizer_block(const hx_lm_config& c) { return c.vocab == kBpeVocabulary; }

size_t encoded_bytes(const hx_lm_config& c, const std::string& kind, const std::string& hash) {
    size_t n = 11 + 8 * 4;
    if (tokenizer_block(c)) n += 4 + kind.size() + 4 + hash.size();
    const auto r = registry(c);
    size_t reg = 4;
    for (const auto& e : r) reg += 4 + e.name.size() + 8 + e.count * 4;
    return n + 3 * reg;
}

struct Writer {
    uint8_t* p;
    void u32(uint32_t v) { for (int s = 24; s >= 0; s -= 8) *p++ = uint8_t(v >> s); }
    void u64(uint64_t v) { for (int s = 56; s >= 0; s -= 8) *p++ = uint8_t(v >> s); }
    void bytes(const void* src, size_t n) { std::memcpy(p, src, n); p += n; }
};

struct Reader {
    const uint8_t* p;
    const uint8_t* end;
    size_t left() const { return size_t(end - p); }
    uint32_t u32() {
        if (left() < 4) fail(HX_ERR_ARGUMENT, "NPRT_CACHE_TRUNCATED_U32");
        uint32_t v = 0;
        for (int i = 0; i < 4; ++i) v = (v << 8) | *p++;
        return v;
    }
    uint64_t u64() {
        if (left() < 8) fail(HX_ERR_ARGUMENT, "NPRT_CACHE_TRUNCATED_U64");
        uint64_t v = 0;
        for (int i = 0; i < 8; ++i) v = (v << 8) | *p++;
        return v;
    }
    bool take(void* dst, size_t n) {
        if (left() < n) { p = end; return false; }
        if (dst) std::memcpy(dst, p, n);
        p += n;
        return true;
    }
};

std::string str_or_empty(const char* s) { return s ? std::string(s) : std::string(); }

void encode(const hx_lm_config& c, uint32_t seed, uint32_t step, const std::string& kind, const std::string& hash,
            const float* params, const float* m, const float* v, std::vector<uint8_t>& out) {
    const auto r = registry(c);
    const uint64_t n = total(r);
    require(params && m && v, HX_ERR_ARGUMENT, "NPRT_CKPT_WRITE_REFUSED: null state buffer");
    require(step != 0, HX_ERR_ARGUMENT, "NPRT_CKPT_WRITE_REFUSED: step 0 is not a resumable state");
    require(all_finite(params, n) && all_finite(m, n) && all_finite(v, n), HX_ERR_ARGUMENT,
            "NPRT_CKPT_WRITE_REFUSED: non-finite training state");
    if (tokenizer_block(c))
        require(kind == "byte_bpe" && hash.size() == 71 && hash.compare(0, 7, "sha256:") == 0, HX_ERR_ARGUMENT,
                "NPRT_CKPT_WRITE_REFUSED: vocabulary 1024 needs tokenizer kind byte_bpe and a sha256: hash of 71 chars");
    else
        require(kind.empty() && hash.empty(), HX_ERR_ARGUMENT,
                "NPRT_CKPT_WRITE_REFUSED: a tokenizer identity is written only at vocabulary 1024");
    out.resize(encoded_bytes(c, kind, hash));
    Writer w{out.data()};
    w.bytes(tokenizer_block(c) ? "NPRTCKPTV3\n" : "NPRTCKPTV2\n", 11);
    for (uint32_t x : {c.vocab, c.tokens, c.dim, c.ffn, c.layers, c.heads, seed, step}) w.u32(x);
    if (tokenizer_block(c)) {
        w.u32(uint32_t(kind.size()));
        w.bytes(kind.data(), kind.size());
        w.u32(uint32_t(hash.size()));
        w.bytes(hash.data(), hash.size());
    }
    for (const float* src : {params, m, v}) {
        w.u32(uint32_t(r.size()));
        uint64_t off = 0;
        for (const auto& e : r) {
            w.u32(uint32_t(e.name.size()));
            w.bytes(e.name.data(), e.name.size());
            w.u64(e.count);
            w.bytes(src + off, e.count * 4);
            off += e.count;
        }
    }
}

void decode(const hx_lm_config& c, uint32_t expected_seed, const std::string& expected_hash, const uint8_t* data,
            size_t size, hx_nprt_info* info, float* params, float* m, float* v) {
    require(data != nullptr, HX_ERR_ARGUMENT, "NPRT_CKPT_OPEN_FAILED");
    if (uint64_t(size) > kNprtMaxBytes) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_SIZE_INVALID");
    hx_nprt_info out{};
    out.finite = 1;
    Reader in{data, data + size};
    char magic[11] = {};
    const bool got_magic = in.take(magic, 11);
    const bool v1 = got_magic && std::memcmp(magic, "NPRTCKPTV1\n", 11) == 0;
    const bool v2 = got_magic && std::memcmp(magic, "NPRTCKPTV2\n", 11) == 0;
    const bool v3 = got_magic && std::memcmp(magic, "NPRTCKPTV3\n", 11) == 0;
    if (!v1 && !v2 && !v3) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_MAGIC");
    out.version = v3 ? 3 : v2 ? 2 : 1;
    const uint32_t vocab = in.u32(), tokens = in.u32(), dim = in.u32(), ffn = in.u32(), layers = in.u32(),
                   heads = in.u32();
    out.seed = in.u32();
    out.step = in.u32();
    if (v3) {
        const uint32_t kind_len = in.u32();
        if (kind_len == 0 || kind_len > 32) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_TOKENIZER_KIND_LENGTH");
        std::string kind(kind_len, '\0');
        in.take(&kind[0], kind_len);  // a short read leaves the next u32 read to fail
        const uint32_t hash_len = in.u32();
        if (hash_len != 71) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_TOKENIZER_HASH_LENGTH");
        std::string hash(71, '\0');
        const bool ok_hash = in.take(&hash[0], 71);
        if (!ok_hash || kind != "byte_bpe" || hash.compare(0, 7, "sha256:") != 0)
            fail(HX_ERR_ARGUMENT, "NPRT_CKPT_TOKENIZER_IDENTITY");
        std::snprintf(out.tokenizer_hash, sizeof out.tokenizer_hash, "%s", hash.c_str());
    }
    const uint32_t reg_count = in.u32();
    if (vocab != c.vocab || tokens != c.tokens || dim != c.dim || ffn != c.ffn || layers != c.layers ||
        heads != c.heads)
        fail(HX_ERR_ARGUMENT, "NPRT_CKPT_CONFIG_MISMATCH");
    if (out.seed != expected_seed) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_SEED_MISMATCH");
    if (c.vocab == kBpeVocabulary) {
        if (!v3) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_V3_REQUIRED_FOR_BPE");
        if (expected_hash.empty() || expected_hash != out.tokenizer_hash)
            fail(HX_ERR_ARGUMENT, "NPRT_CKPT_TOKENIZER_HASH_MISMATCH");
    } else if (v3) {
        fail(HX_ERR_ARGUMENT, "NPRT_CKPT_V3_REQUIRES_BPE_MODEL");
    }
    if (out.step == 0 || out.step >= 1000000) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_STEP_INVALID");
    const auto r = registry(c);
    if (reg_count != r.size()) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_REGISTRY_COUNT_MISMATCH");
    uint64_t hash = kFnvOffset;
    auto fnv = [&hash](const void* src, size_t n) {
        const uint8_t* b = static_cast<const uint8_t*>(src);
        for (size_t i = 0; i < n; ++i) {
            hash ^= b[i];
            hash *= kFnvPrime;
        }
    };
    auto read_registry = [&](float* dst, bool moments) {
        if (moments) {
            const uint32_t count = in.u32();
            if (count != r.size()) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_ADAM_REGISTRY_COUNT");
        }
        uint64_t off = 0;
        for (const auto& e : r) {
            const uint32_t name_len = in.u32();
            if (name_len == 0 || name_len > 256) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_NAME_LENGTH");
            std::string name(name_len, '\0');
            if (!in.take(&name[0], name_len)) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_NAME_TRUNCATED");
            const uint64_t count = in.u64();
            if (moments) {
                if (name != e.name || count != e.count || count > 100000000ull)
                    fail(HX_ERR_ARGUMENT, "NPRT_CKPT_ADAM_REGISTRY_IDENTITY");
            } else {
                if (name != e.name) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_REGISTRY_ORDER_MISMATCH");
                if (count != e.count || count > 100000000ull) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_ELEMENT_COUNT_MISMATCH");
            }
            const uint8_t* values = in.p;
            if (!in.take(nullptr, count * 4)) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_VALUES_TRUNCATED");
            for (uint64_t i = 0; i < count; ++i) {
                float f;
                std::memcpy(&f, values + 4 * i, 4);
                if (!std::isfinite(f)) out.finite = 0;
            }
            if (!moments) {
                fnv(e.name.data(), e.name.size());
                fnv(&count, sizeof count);
                fnv(values, count * 4);
            }
            if (dst) std::memcpy(dst + off, values, count * 4);
            off += count;
        }
    };
    read_registry(params, false);
    if (v2 || v3) {
        out.has_adam = 1;
        read_registry(m, true);
        read_registry(v, true);
    }
    if (in.left() != 0) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_TRAILING_BYTES");
    out.parameter_count = total(r);
    std::snprintf(out.parameter_hash, sizeof out.parameter_hash, "fnv1a64:%016llx", (unsigned long long)hash);
    if (info) *info = out;
}

void copy_error(const std::string& msg, char* err, size_t cap) {
    if (err && cap) std::snprintf(err, cap, "%s", msg.c_str());
}

// Runs a host-only codec call: no runtime, so the message goes to `err`.
template <class F>
int codec_guard(char* err, size_t cap, F&& body) {
    try {
        body();
        copy_error("", err, cap);
        return HX_OK;
    } catch (const Error& e) {
        copy_error(e.message, err, cap);
        return e.code;
    } catch (const std::bad_alloc&) {
        copy_error("host allocation failed", err, cap);
        return HX_ERR_MEMORY;
    }
}

std::vector<uint8_t> read_file(const char* path) {
    FILE* f = path ? std::fopen(path, "rb") : nullptr;
    if (!f) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_OPEN_FAILED");
    if (std::fseek(f, 0, SEEK_END) != 0) {
        std::fclose(f);
        fail(HX_ERR_ARGUMENT, "NPRT_CKPT_OPEN_FAILED");
    }
    const long n = std::ftell(f);
    if (n < 0 || uint64_t(n) > kNprtMaxBytes) {
        std::fclose(f);
        fail(HX_ERR_ARGUMENT, "NPRT_CKPT_SIZE_INVALID");
    }
    std::vector<uint8_t> buf(static_cast<size_t>(n));
    std::rewind(f);
    const size_t got = buf.empty() ? 0 : std::fread(buf.data(), 1, buf.size(), f);
    std::fclose(f);
    if (got != buf.size()) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_OPEN_FAILED");
    return buf;
}

// Writes `bytes` to "<path>.tmp", then renames it over `path`, so a reader
// never sees a partial file under the final name.
void write_atomic(const std::string& path, const std::vector<uint8_t>& bytes) {
    const std::string tmp = path + ".tmp";
    std::remove(tmp.c_str());
    FILE* f = std::fopen(tmp.c_str(), "wb");
    if (!f) fail(HX_ERR_ARGUMENT, "NPRT_CKPT_WRITE_FAILED: cannot open " + tmp);
    const size_t put = bytes.empty() ? 0 : std::fwrite(bytes.data(), 1, bytes.size(), f);
    const bool ok = put == bytes.size() && std::fflush(f) == 0;
    if (std::fclose(f) != 0 || !ok) {
        std::remove(tmp.c_str());
        fail(HX_ERR_ARGUMENT, "NPRT_CKPT_WRITE_FAILED: short write to " + tmp);
    }
    if (std::rename(tmp.c_str(), path.c_str()) != 0) {
        std::remove(tmp.c_str());
        fail(HX_ERR_ARGUMENT, "NPRT_CKPT_WRITE_FAILED: cannot replace " + path);
    }
}

uint64_t splitmix(uint64_t x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

}  // namespace
}  // namespace hx

using namespace hx;

extern "C" {

size_t hx_nprt_encoded_bytes(const hx_lm_config* config, const char* tokenizer_kind, const char* tokenizer_hash) {
    if (!config) return 0;
    return encoded_bytes(*config, str_or_empty(tokenizer_kind), str_or_empty(tokenizer_hash));
}

int hx_nprt_encode(const hx_lm_config* config, uint32_t seed, uint32_t step, const char* tokenizer_kind,
                   const char* tokenizer_hash, const float* params, const float* adam_m, const float* adam_v,
                   uint8_t* out, size_t capacity, size_t* written, char* error, size_t error_capacity) {
    return codec_guard(error, error_capacity, [&] {
        require(config && out && written, HX_ERR_ARGUMENT, "NPRT_CKPT_WRITE_REFUSED: null argument");
        std::vector<uint8_t> bytes;
        encode(*config, seed, step, str_or_empty(tokenizer_kind), str_or_empty(tokenizer_hash), params, adam_m,
               adam_v, bytes);
        require(bytes.size() <= capacity, HX_ERR_ARGUMENT, "NPRT_CKPT_WRITE_REFUSED: output buffer too small");
        std::memcpy(out, bytes.data(), bytes.size());
        *written = bytes.size();
    });
}

int hx_nprt_decode(const hx_lm_config* config, uint32_t expected_seed, const char* expected_tokenizer_hash,
                   const uint8_t* data, size_t size, hx_nprt_info* info, float* params, float* adam_m,
                   float* adam_v, char* error, size_t error_capacity) {
    return codec_guard(error, error_capacity, [&] {
        require(config != nullptr, HX_ERR_ARGUMENT, "NPRT_CKPT_CONFIG_MISMATCH");
        decode(*config, expected_seed, str_or_empty(expected_tokenizer_hash), data, size, info, params, adam_m,
               adam_v);
    });
}

int hx_nprt_checkpoint_name(uint32_t seed, uint32_t layers, uint32_t tokens, uint32_t dimension,
                            uint32_t feed_forward_dimension, uint32_t step, char* out, size_t capacity) {
    if (!out || capacity == 0) return HX_ERR_ARGUMENT;
    std::string name = "htp-seed" + std::to_string(seed) + "-l" + std::to_string(layers);
    if (!(tokens == 32 && dimension == 32 && feed_forward_dimension == 32))
        name += "-t" + std::to_string(tokens) + "-d" + std::to_string(dimension) + "-f" +
                std::to_string(feed_forward_dimension);
    name += "-step" + std::to_string(step) + ".ckpt";
    if (name.size() + 1 > capacity) return HX_ERR_ARGUMENT;
    std::memcpy(out, name.c_str(), name.size() + 1);
    return HX_OK;
}

int hx_nprt_training_order(uint64_t record_count, uint32_t steps, uint32_t batch, uint64_t* out) {
    if (!out || record_count == 0) return HX_ERR_ARGUMENT;
    uint64_t state = 20260806;
    const uint64_t n = uint64_t(steps) * batch;
    for (uint64_t i = 0; i < n; ++i) {
        state = splitmix(state + i);
        out[i] = state % record_count;
    }
    return HX_OK;
}

int hx_lm_checkpoint_save(hx_runtime* rt, const char* path, uint32_t seed, uint32_t step,
                          const char* tokenizer_kind, const char* tokenizer_hash) {
    return hx_guard(rt, [&] {
        require(path && *path, HX_ERR_ARGUMENT, "NPRT_CKPT_WRITE_FAILED: empty path");
        hx_lm_config cfg{};
        uint32_t opt = 0;
        require(lm_prepared_config(rt, &cfg, &opt), HX_ERR_STATE, "generalized tiny training graph not prepared");
        require(opt == HX_OPT_ADAM, HX_ERR_UNSUPPORTED,
                "NPRT_CKPT_WRITE_REFUSED: the format carries Adam moments only; Muon momentum buffers would be lost");
        const size_t n = hx_lm_param_count(&cfg);
        std::vector<float> p(n), m(n), v(n);
        if (hx_lm_state_download(rt, p.data(), m.data(), v.data(), nullptr, n) != HX_OK)
            fail(HX_ERR_STATE, rt->last_error);
        std::vector<uint8_t> bytes;
        encode(cfg, seed, step, str_or_empty(tokenizer_kind), str_or_empty(tokenizer_hash), p.data(), m.data(),
               v.data(), bytes);
        write_atomic(path, bytes);
    });
}

int hx_lm_checkpoint_resume(hx_runtime* rt, const char* path, uint32_t expected_seed, uint32_t expected_step,
                            const char* tokenizer_hash, hx_nprt_info* info) {
    return hx_guard(rt, [&] {
        hx_lm_config cfg{};
        uint32_t opt = 0;
        require(lm_prepared_config(rt, &cfg, &opt), HX_ERR_STATE, "generalized tiny training graph not prepared");
        require(opt == HX_OPT_ADAM, HX_ERR_UNSUPPORTED,
                "RESUME_OPTIMIZER: the format carries Adam moments only; resume needs the Adam optimizer");
        const size_t n = hx_lm_param_count(&cfg);
        std::vector<float> p(n), m(n), v(n);
        hx_nprt_info got{};
        try {
            const auto bytes = read_file(path);
            decode(cfg, expected_seed, str_or_empty(tokenizer_hash), bytes.data(), bytes.size(), &got, p.data(),
                   m.data(), v.data());
        } catch (const Error& e) {
            fail(e.code, "RESUME_CHECKPOINT_DECODE: " + e.message);
        }
        if ((expected_step != 0 && got.step != expected_step) || !got.finite)
            fail(HX_ERR_ARGUMENT, "RESUME_CHECKPOINT_IDENTITY: resume checkpoint step/finiteness mismatch");
        if (!got.has_adam)
            fail(HX_ERR_ARGUMENT,
                 "RESUME_ADAM_STATE_MISSING: NPRTCKPTV1 has no Adam moments; canonical resume requires NPRTCKPTV2");
        if (hx_lm_state_upload(rt, p.data(), m.data(), v.data(), nullptr, n) != HX_OK) fail(HX_ERR_STATE, rt->last_error);
        if (info) *info = got;
    });
}

}  // extern "C"
