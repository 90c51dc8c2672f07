// Official checkpoint loading: safetensors files (an 8-byte little-endian header size, a JSON header
// {name: {"dtype", "shape", "data_offsets"}, "__metadata__": {...}}, then the raw little-endian tensor data)
// read straight into the resident models, in place of the reference's packaging step (tools/
// build_dit_weights.py, tools/build_text_weights.py, tools/export_vae.py write ncnn .bin files from the same
// safetensors). Also text_embeddings (src/text_encoder.cpp:48-75) over the reference's raw BF16 table or the
// checkpoint's embed_tokens tensor.
#include "capi_internal.h"
#include "ernie_cuda.h"
#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace
{
int fail_weights(const std::string &message) { return ernie_b200::capi::fail(ERNIE_CUDA_ERROR, message); }

struct Entry
{
    std::string dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;
};

// Minimal JSON reader for the safetensors header: objects, arrays, strings, integers (and skipped values).
class Json
{
  public:
    explicit Json(const std::string &text) : s_(text) {}
    std::map<std::string, Entry> header()
    {
        std::map<std::string, Entry> out;
        expect('{');
        if (peek() == '}')
        {
            ++i_;
            return out;
        }
        while (true)
        {
            const std::string name = string();
            expect(':');
            if (name == "__metadata__") skip();
            else
            {
                if (out.count(name)) throw std::runtime_error("Duplicate tensor " + name);
                out[name] = entry(name);
            }
            if (peek() == ',')
            {
                ++i_;
                continue;
            }
            expect('}');
            break;
        }
        ws();
        if (i_ != s_.size()) throw std::runtime_error("Trailing bytes after the safetensors header");
        return out;
    }

  private:
    const std::string &s_;
    size_t i_ = 0;
    void ws()
    {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\t' || s_[i_] == '\n' || s_[i_] == '\r')) ++i_;
    }
    char peek()
    {
        ws();
        if (i_ >= s_.size()) throw std::runtime_error("Truncated safetensors header");
        return s_[i_];
    }
    void expect(char c)
    {
        if (peek() != c) throw std::runtime_error(std::string("Malformed safetensors header: expected ") + c);
        ++i_;
    }
    std::string string()
    {
        expect('"');
        std::string out;
        while (i_ < s_.size() && s_[i_] != '"')
        {
            if (s_[i_] == '\\')
            {
                if (++i_ >= s_.size()) break;
                const char e = s_[i_];
                if (e == 'u') throw std::runtime_error("Unicode escapes are not used in tensor names");
                out += e == 'n' ? '\n' : e == 't' ? '\t' : e;
            }
            else out += s_[i_];
            ++i_;
        }
        if (i_ >= s_.size()) throw std::runtime_error("Unterminated string in safetensors header");
        ++i_;
        return out;
    }
    int64_t integer()
    {
        ws();
        size_t start = i_;
        if (i_ < s_.size() && s_[i_] == '-') ++i_;
        while (i_ < s_.size() && s_[i_] >= '0' && s_[i_] <= '9') ++i_;
        if (start == i_ || (s_[start] == '-' && i_ == start + 1)) throw std::runtime_error("Expected an integer");
        return std::stoll(s_.substr(start, i_ - start));
    }
    std::vector<int64_t> int_array()
    {
        std::vector<int64_t> out;
        expect('[');
        if (peek() == ']')
        {
            ++i_;
            return out;
        }
        while (true)
        {
            out.push_back(integer());
            if (peek() == ',')
            {
                ++i_;
                continue;
            }
            expect(']');
            return out;
        }
    }
    void skip()
    {
        const char c = peek();
        if (c == '"') string();
        else if (c == '{' || c == '[')
        {
            const char close = c == '{' ? '}' : ']';
            ++i_;
            if (peek() == close)
            {
                ++i_;
                return;
            }
            while (true)
            {
                if (c == '{')
                {
                    string();
                    expect(':');
                }
                skip();
                if (peek() == ',')
                {
                    ++i_;
                    continue;
                }
                expect(close);
                return;
            }
        }
        else
        {
            while (i_ < s_.size() && s_[i_] != ',' && s_[i_] != '}' && s_[i_] != ']') ++i_;
        }
    }
    Entry entry(const std::string &name)
    {
        Entry e;
        bool dtype = false, shape = false, offsets = false;
        expect('{');
        while (true)
        {
            const std::string key = string();
            expect(':');
            if (key == "dtype")
            {
                e.dtype = string();
                dtype = true;
            }
            else if (key == "shape")
            {
                e.shape = int_array();
                shape = true;
            }
            else if (key == "data_offsets")
            {
                const auto o = int_array();
                if (o.size() != 2 || o[0] < 0 || o[1] < o[0]) throw std::runtime_error("Invalid data_offsets of " + name);
                e.begin = static_cast<uint64_t>(o[0]);
                e.end = static_cast<uint64_t>(o[1]);
                offsets = true;
            }
            else skip();
            if (peek() == ',')
            {
                ++i_;
                continue;
            }
            expect('}');
            break;
        }
        if (!dtype || !shape || !offsets) throw std::runtime_error("Incomplete tensor entry " + name);
        for (int64_t d : e.shape)
            if (d < 0) throw std::runtime_error("Negative dimension in " + name);
        return e;
    }
};

size_t dtype_bytes(const std::string &dtype)
{
    if (dtype == "BF16" || dtype == "F16") return 2;
    if (dtype == "F32") return 4;
    return 0;
}

class SafeFile
{
  public:
    explicit SafeFile(const std::string &path) : path_(path), in_(path, std::ios::binary)
    {
        if (!in_) throw std::runtime_error("Cannot open " + path);
        in_.seekg(0, std::ios::end);
        const uint64_t size = static_cast<uint64_t>(in_.tellg());
        in_.seekg(0);
        unsigned char raw[8];
        if (size < 8 || !in_.read(reinterpret_cast<char *>(raw), 8)) throw std::runtime_error("Truncated safetensors file " + path);
        uint64_t header = 0;
        for (int b = 7; b >= 0; --b) header = (header << 8) | raw[b];
        if (header > 100u * 1024 * 1024 || 8 + header > size) throw std::runtime_error("Invalid safetensors header size in " + path);
        std::string text(header, '\0');
        if (!in_.read(&text[0], static_cast<std::streamsize>(header))) throw std::runtime_error("Truncated header in " + path);
        entries_ = Json(text).header();
        data_ = 8 + header;
        for (const auto &[name, e] : entries_)
        {
            uint64_t count = 1;
            for (int64_t d : e.shape) count *= static_cast<uint64_t>(d);
            const size_t bytes = dtype_bytes(e.dtype);
            if (bytes && e.end - e.begin != count * bytes) throw std::runtime_error("Byte count differs from the shape: " + name);
            if (data_ + e.end > size) throw std::runtime_error("Tensor data past the end of the file: " + name);
        }
    }
    const std::map<std::string, Entry> &entries() const { return entries_; }
    const std::string &path() const { return path_; }
    // The tensor as FP32 (BF16 / F16 / F32 sources), after checking the shape; non-finite values rejected.
    std::vector<float> read_f32(const std::string &name, const std::vector<int64_t> &shape)
    {
        const Entry &e = entry(name, shape);
        std::vector<float> out(count(e));
        if (e.dtype == "F32")
        {
            read(e, out.data(), out.size() * 4);
        }
        else
        {
            std::vector<uint16_t> raw(out.size());
            read(e, raw.data(), raw.size() * 2);
            for (size_t i = 0; i < raw.size(); ++i) out[i] = widen(raw[i], e.dtype == "BF16");
        }
        for (float v : out)
            if (!std::isfinite(v)) throw std::runtime_error("Non-finite weight: " + name);
        return out;
    }
    // BF16 bits of a BF16 tensor (the DiT and text GEMM weights stay BF16, losslessly).
    std::vector<uint16_t> read_bf16(const std::string &name, const std::vector<int64_t> &shape)
    {
        const Entry &e = entry(name, shape);
        if (e.dtype != "BF16") throw std::runtime_error("Expected BF16: " + name + " is " + e.dtype);
        std::vector<uint16_t> out(count(e));
        read(e, out.data(), out.size() * 2);
        for (uint16_t b : out)
            if ((b & 0x7F80u) == 0x7F80u) throw std::runtime_error("Non-finite weight: " + name);
        return out;
    }
    // rows [row, row + 1) of a 2D tensor as FP32
    void read_row_f32(const std::string &name, uint64_t row, float *dst)
    {
        const Entry &e = entries_.at(name);
        const uint64_t width = static_cast<uint64_t>(e.shape.at(1)), elem = dtype_bytes(e.dtype);
        std::vector<unsigned char> raw(width * elem);
        in_.seekg(static_cast<std::streamoff>(data_ + e.begin + row * width * elem));
        if (!in_.read(reinterpret_cast<char *>(raw.data()), static_cast<std::streamsize>(raw.size())))
            throw std::runtime_error("Embedding row read failed");
        for (uint64_t j = 0; j < width; ++j)
        {
            if (elem == 4) std::memcpy(dst + j, &raw[j * 4], 4);
            else dst[j] = widen(static_cast<uint16_t>(raw[j * 2] | (raw[j * 2 + 1] << 8)), e.dtype == "BF16");
        }
    }

  private:
    std::string path_;
    std::ifstream in_;
    std::map<std::string, Entry> entries_;
    uint64_t data_ = 0;

    static uint64_t count(const Entry &e)
    {
        uint64_t n = 1;
        for (int64_t d : e.shape) n *= static_cast<uint64_t>(d);
        return n;
    }
    static float widen(uint16_t v, bool bf16)
    {
        if (bf16)
        {
            const uint32_t bits = static_cast<uint32_t>(v) << 16;
            float f;
            std::memcpy(&f, &bits, 4);
            return f;
        }
        // IEEE half
        const uint32_t sign = (v >> 15) & 1u, exp = (v >> 10) & 31u, man = v & 1023u;
        float f;
        if (exp == 0) f = std::ldexp(static_cast<float>(man), -24);
        else if (exp == 31) f = man ? NAN : INFINITY;
        else f = std::ldexp(static_cast<float>(man | 1024u), static_cast<int>(exp) - 25);
        return sign ? -f : f;
    }
    const Entry &entry(const std::string &name, const std::vector<int64_t> &shape)
    {
        const auto it = entries_.find(name);
        if (it == entries_.end()) throw std::runtime_error("Missing tensor " + name);
        if (!dtype_bytes(it->second.dtype)) throw std::runtime_error("Unsupported dtype " + it->second.dtype + ": " + name);
        std::vector<int64_t> have = it->second.shape, want = shape;
        // a 1x1 convolution's trailing unit dimensions are a linear layer's weight
        while (have.size() > want.size() && have.back() == 1) have.pop_back();
        if (have != want) throw std::runtime_error("Unexpected shape of " + name);
        return it->second;
    }
    void read(const Entry &e, void *dst, size_t bytes)
    {
        in_.seekg(static_cast<std::streamoff>(data_ + e.begin));
        if (!in_.read(static_cast<char *>(dst), static_cast<std::streamsize>(bytes)))
            throw std::runtime_error("Tensor read failed in " + path_);
    }
};

// The tensor `name` from whichever of the files holds it (sharded checkpoints).
struct Checkpoint
{
    std::vector<std::unique_ptr<SafeFile>> files;
    Checkpoint(const char *const *paths, int count)
    {
        if (!paths || count < 1) throw std::invalid_argument("No safetensors files");
        for (int i = 0; i < count; ++i)
        {
            if (!paths[i]) throw std::invalid_argument("Null file name");
            files.push_back(std::make_unique<SafeFile>(paths[i]));
        }
    }
    SafeFile &holder(const std::string &name)
    {
        for (auto &f : files)
            if (f->entries().count(name)) return *f;
        throw std::runtime_error("Missing tensor " + name);
    }
    std::vector<float> f32(const std::string &name, const std::vector<int64_t> &shape)
    {
        return holder(name).read_f32(name, shape);
    }
    std::vector<uint16_t> bf16(const std::string &name, const std::vector<int64_t> &shape)
    {
        return holder(name).read_bf16(name, shape);
    }
};

template <class F> int guarded(F &&f)
{
    try
    {
        return f();
    }
    catch (const std::exception &e)
    {
        return fail_weights(e.what());
    }
}

// the upload calls record their own message in the thread's last error
int forward(int rc, const char *) { return rc; }
} // namespace

extern "C" int ernie_cuda_safetensors_count(const char *path, int *count)
{
    return guarded([&] {
        if (!path || !count) return fail_weights("null argument");
        SafeFile f(path);
        *count = static_cast<int>(f.entries().size());
        return ERNIE_CUDA_OK;
    });
}

extern "C" int ernie_cuda_safetensors_entry(const char *path, int index, char *name, size_t name_bytes, char *dtype,
                                            int64_t *dims, int *ndim)
{
    return guarded([&] {
        if (!path || !name || !dtype || !dims || !ndim) return fail_weights("null argument");
        SafeFile f(path);
        if (index < 0 || index >= static_cast<int>(f.entries().size())) return fail_weights("Entry index out of range");
        auto it = f.entries().begin();
        std::advance(it, index);
        if (it->first.size() + 1 > name_bytes || it->second.shape.size() > 8) return fail_weights("Buffer too small");
        std::memcpy(name, it->first.c_str(), it->first.size() + 1);
        std::strncpy(dtype, it->second.dtype.c_str(), 7);
        dtype[7] = '\0';
        *ndim = static_cast<int>(it->second.shape.size());
        for (size_t d = 0; d < it->second.shape.size(); ++d) dims[d] = it->second.shape[d];
        return ERNIE_CUDA_OK;
    });
}

extern "C" int ernie_cuda_model_load_safetensors(ernie_cuda_model *model, int num_blocks, const char *const *files,
                                                 int count, int with_heads)
{
    return guarded([&] {
        if (!model || num_blocks < 0) return fail_weights("null model or negative block count");
        Checkpoint ck(files, count);
        const int64_t H = 4096, F = 12288;
        for (int b = 0; b < num_blocks; ++b)
        {
            const std::string p = "layers." + std::to_string(b) + ".";
            const auto wq = ck.bf16(p + "self_attention.to_q.weight", {H, H});
            const auto wk = ck.bf16(p + "self_attention.to_k.weight", {H, H});
            const auto wv = ck.bf16(p + "self_attention.to_v.weight", {H, H});
            const auto wo = ck.bf16(p + "self_attention.to_out.0.weight", {H, H});
            const auto wup = ck.bf16(p + "mlp.up_proj.weight", {F, H});
            const auto wgate = ck.bf16(p + "mlp.gate_proj.weight", {F, H});
            const auto wfc2 = ck.bf16(p + "mlp.linear_fc2.weight", {H, F});
            const auto gsa = ck.f32(p + "adaLN_sa_ln.weight", {H});
            const auto gmlp = ck.f32(p + "adaLN_mlp_ln.weight", {H});
            const auto gq = ck.f32(p + "self_attention.norm_q.weight", {128});
            const auto gk = ck.f32(p + "self_attention.norm_k.weight", {128});
            const ernie_cuda_block_weights w{wq.data(),   wk.data(),  wv.data(),   wo.data(), wup.data(), wgate.data(),
                                             wfc2.data(), gsa.data(), gmlp.data(), gq.data(), gk.data()};
            const int rc = forward(ernie_cuda_model_upload_block(model, b, &w), "upload block");
            if (rc != ERNIE_CUDA_OK) return rc;
        }
        if (!with_heads) return ERNIE_CUDA_OK;
        const auto xw = ck.bf16("x_embedder.proj.weight", {H, 128});
        const auto xb = ck.f32("x_embedder.proj.bias", {H});
        const auto tp = ck.bf16("text_proj.weight", {H, 3072});
        const auto t1w = ck.bf16("time_embedding.linear_1.weight", {H, H});
        const auto t1b = ck.f32("time_embedding.linear_1.bias", {H});
        const auto t2w = ck.bf16("time_embedding.linear_2.weight", {H, H});
        const auto t2b = ck.f32("time_embedding.linear_2.bias", {H});
        const auto aw = ck.bf16("adaLN_modulation.1.weight", {6 * H, H});
        const auto ab = ck.f32("adaLN_modulation.1.bias", {6 * H});
        const auto fnw = ck.bf16("final_norm.linear.weight", {2 * H, H});
        const auto fnb = ck.f32("final_norm.linear.bias", {2 * H});
        const auto fw = ck.bf16("final_linear.weight", {128, H});
        const auto fb = ck.f32("final_linear.bias", {128});
        const ernie_cuda_head_weights h{xw.data(), xb.data(),  tp.data(),  t1w.data(), t1b.data(), t2w.data(), t2b.data(),
                                        aw.data(), ab.data(),  fnw.data(), fnb.data(), fw.data(),  fb.data()};
        return forward(ernie_cuda_model_upload_heads(model, &h), "upload heads");
    });
}

namespace
{
// Mistral decoder layers 0..num_layers-1 under `prefix` + "{l}." into the text model.
int load_mistral_layers(ernie_cuda_text_model *model, int num_layers, Checkpoint &ck, const std::string &prefix)
{
        const int64_t H = 3072, Q = 4096, KV = 1024, F = 9216;
        for (int l = 0; l < num_layers; ++l)
        {
            const std::string p = prefix + std::to_string(l) + ".";
            const auto wq = ck.bf16(p + "self_attn.q_proj.weight", {Q, H});
            const auto wk = ck.bf16(p + "self_attn.k_proj.weight", {KV, H});
            const auto wv = ck.bf16(p + "self_attn.v_proj.weight", {KV, H});
            const auto wo = ck.bf16(p + "self_attn.o_proj.weight", {H, Q});
            const auto wg = ck.bf16(p + "mlp.gate_proj.weight", {F, H});
            const auto wu = ck.bf16(p + "mlp.up_proj.weight", {F, H});
            const auto wd = ck.bf16(p + "mlp.down_proj.weight", {H, F});
            const auto ga = ck.f32(p + "input_layernorm.weight", {H});
            const auto gm = ck.f32(p + "post_attention_layernorm.weight", {H});
            const ernie_cuda_text_layer_weights w{wq.data(), wk.data(), wv.data(), wo.data(), wg.data(),
                                                  wu.data(), wd.data(), ga.data(), gm.data()};
            const int rc = forward(ernie_cuda_text_model_upload_layer(model, l, &w), "upload text layer");
            if (rc != ERNIE_CUDA_OK) return rc;
        }
        return ERNIE_CUDA_OK;
}
} // namespace

extern "C" int ernie_cuda_text_model_load_safetensors(ernie_cuda_text_model *model, int num_layers,
                                                      const char *const *files, int count)
{
    return guarded([&] {
        if (!model || num_layers < 1) return fail_weights("null model or no layers");
        Checkpoint ck(files, count);
        return load_mistral_layers(model, num_layers, ck, "language_model.model.layers.");
    });
}

extern "C" int ernie_cuda_pe_model_load_safetensors(ernie_cuda_text_model *model, int num_layers,
                                                    const char *const *files, int count)
{
    return guarded([&] {
        if (!model || num_layers < 1) return fail_weights("null model or no layers");
        Checkpoint ck(files, count);
        const int rc = load_mistral_layers(model, num_layers, ck, "model.layers.");
        if (rc != ERNIE_CUDA_OK) return rc;
        // the LM head is tied to the embeddings in the official config (tools/build_pe_model.py:68-73)
        std::string head = "lm_head.weight";
        bool found = false;
        for (auto &f : ck.files) found = found || f->entries().count(head) > 0;
        if (!found) head = "model.embed_tokens.weight";
        const auto norm = ck.f32("model.norm.weight", {3072});
        const auto w = ck.bf16(head, {131072, 3072});
        return forward(ernie_cuda_text_model_upload_head(model, norm.data(), w.data()), "upload PE head");
    });
}

extern "C" int ernie_cuda_vae_load_safetensors(ernie_cuda_vae *vae, const char *const *files, int count)
{
    return guarded([&] {
        if (!vae) return fail_weights("null VAE");
        Checkpoint ck(files, count);
        int n = 0;
        ernie_cuda_vae_tensor_count(&n);
        for (int i = 0; i < n; ++i)
        {
            char name[128];
            int dims[4] = {0, 0, 0, 0}, nd = 0;
            ernie_cuda_vae_tensor_info(i, name, sizeof(name), dims, &nd);
            const auto v = ck.f32(name, std::vector<int64_t>(dims, dims + nd));
            const int rc = forward(ernie_cuda_vae_upload(vae, name, v.data(), v.size()), "upload VAE tensor");
            if (rc != ERNIE_CUDA_OK) return rc;
        }
        return ERNIE_CUDA_OK;
    });
}

extern "C" int ernie_cuda_vae_encoder_load_safetensors(ernie_cuda_vae_encoder *encoder, const char *const *files,
                                                       int count)
{
    return guarded([&] {
        if (!encoder) return fail_weights("null VAE encoder");
        Checkpoint ck(files, count);
        int n = 0;
        ernie_cuda_vae_encoder_tensor_count(&n);
        for (int i = 0; i < n; ++i)
        {
            char name[128];
            int dims[4] = {0, 0, 0, 0}, nd = 0;
            ernie_cuda_vae_encoder_tensor_info(i, name, sizeof(name), dims, &nd);
            const auto v = ck.f32(name, std::vector<int64_t>(dims, dims + nd));
            const int rc = forward(ernie_cuda_vae_encoder_upload(encoder, name, v.data(), v.size()),
                                   "upload VAE encoder tensor");
            if (rc != ERNIE_CUDA_OK) return rc;
        }
        return ERNIE_CUDA_OK;
    });
}

extern "C" int ernie_cuda_text_embeddings(const char *path, const uint32_t *ids, int count, int bucket, float *out)
{
    return guarded([&] {
        if (!path || !ids || !out) return fail_weights("null argument");
        if (bucket < 1 || bucket > 2048) return fail_weights("Text bucket must be in [1,2048]");
        if (count < 1 || count > bucket) return fail_weights("Invalid token IDs or BF16 embedding table size");
        const uint64_t vocab = 131072, width = 3072;
        std::memset(out, 0, static_cast<size_t>(bucket) * width * 4);
        const std::string p(path);
        if (p.size() > 12 && p.compare(p.size() - 12, 12, ".safetensors") == 0)
        {
            SafeFile f(p);
            const std::string name = "language_model.model.embed_tokens.weight";
            const auto it = f.entries().find(name);
            if (it == f.entries().end() || it->second.shape != std::vector<int64_t>{int64_t(vocab), int64_t(width)})
                return fail_weights("Invalid token IDs or BF16 embedding table size");
            for (int i = 0; i < count; ++i)
            {
                if (ids[i] >= vocab) return fail_weights("Token ID outside vocabulary");
                f.read_row_f32(name, ids[i], out + static_cast<size_t>(i) * width);
            }
            return ERNIE_CUDA_OK;
        }
        // the reference's converted table: raw BF16 [131072][3072], only requested rows read
        std::ifstream file(p, std::ios::binary);
        file.seekg(0, std::ios::end);
        if (!file || static_cast<uint64_t>(file.tellg()) != vocab * width * 2)
            return fail_weights("Invalid token IDs or BF16 embedding table size");
        std::vector<unsigned char> row(width * 2);
        for (int i = 0; i < count; ++i)
        {
            if (ids[i] >= vocab) return fail_weights("Token ID outside vocabulary");
            file.seekg(static_cast<std::streamoff>(uint64_t(ids[i]) * width * 2));
            if (!file.read(reinterpret_cast<char *>(row.data()), static_cast<std::streamsize>(row.size())))
                return fail_weights("Embedding row read failed");
            float *target = out + static_cast<size_t>(i) * width;
            for (uint64_t j = 0; j < width; ++j)
            {
                const uint32_t bits = (uint32_t(row[2 * j]) | uint32_t(row[2 * j + 1]) << 8) << 16;
                std::memcpy(&target[j], &bits, 4);
            }
        }
        return ERNIE_CUDA_OK;
    });
}
