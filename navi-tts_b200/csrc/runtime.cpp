#include "runtime.hpp"

#include "../../include/navi_b200.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <set>

namespace navi {

void fail(const std::string & msg, int status) { throw Error(msg, status); }

void cuda_check(cudaError_t e, const char * what, const char * file, int line) {
    if (e == cudaSuccess) return;
    const int st = (e == cudaErrorMemoryAllocation) ? NAVI_E_NOMEM : NAVI_E_CUDA;
    fail(std::string(what) + ": " + cudaGetErrorString(e) + " (" + file + ":" + std::to_string(line) + ")", st);
}

size_t dtype_size(DType d) {
    switch (d) {
        case DType::F32: return 4;
        case DType::F16: return 2;
        case DType::BF16: return 2;
        case DType::I32: return 4;
        case DType::U8: return 1;
    }
    return 0;
}

uint64_t TensorInfo::numel() const {
    uint64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
}

// ---- .navi reader ---------------------------------------------------------------------------------
//
// The file is mapped read-only once; the header is decoded straight from the mapping by a
// cursor that knows where the header ends (data_offset) and names the field and the byte
// offset of whatever does not fit. Byte layout: the reference's docs/navi-format.md:10-47.

namespace {

constexpr uint64_t kPage = 4096;
constexpr uint64_t kPreambleBytes = 32;
constexpr uint32_t kFormatVersion = 1;

class HeaderCursor {
public:
    HeaderCursor(const uint8_t * base, uint64_t end, const std::string & file) : base_(base), end_(end), file_(file) {}

    void limit(uint64_t end) { end_ = end; }

    template <class T> T scalar(const char * field) {
        T v;
        std::memcpy(&v, span(sizeof(T), field), sizeof(T));
        return v;
    }
    std::string text(const char * field) {
        const auto n = scalar<uint32_t>(field);
        const char * p = reinterpret_cast<const char *>(span(n, field));
        return std::string(p, n);
    }

private:
    const uint8_t * span(uint64_t n, const char * field) {
        if (n > end_ - at_)
            fail(file_ + ": " + field + " at header byte " + std::to_string(at_) + " needs " + std::to_string(n) +
                     " bytes, but the header ends at byte " + std::to_string(end_),
                 NAVI_E_FORMAT);
        const uint8_t * p = base_ + at_;
        at_ += n;
        return p;
    }
    const uint8_t * base_;
    uint64_t end_, at_ = 0;
    const std::string & file_;
};

KV decode_value(HeaderCursor & c, const std::string & file, const std::string & key) {
    KV v;
    const auto tag = c.scalar<uint8_t>("hyperparameter type");
    switch (tag) {
        case static_cast<uint8_t>(KV::Type::I64): v.i64 = c.scalar<int64_t>("integer value"); break;
        case static_cast<uint8_t>(KV::Type::F64): v.f64 = c.scalar<double>("float value"); break;
        case static_cast<uint8_t>(KV::Type::STR): v.str = c.text("string value"); break;
        case static_cast<uint8_t>(KV::Type::I64_ARRAY): {
            const auto n = c.scalar<uint32_t>("array length");
            v.arr.resize(n);
            for (auto & x : v.arr) x = c.scalar<int64_t>("array element");
            break;
        }
        default:
            fail(file + ": hyperparameter '" + key + "' has type code " + std::to_string(tag) + ", which version 1 does not define",
                 NAVI_E_FORMAT);
    }
    v.type = static_cast<KV::Type>(tag);
    return v;
}

TensorInfo decode_tensor(HeaderCursor & c, const std::string & file, uint64_t data_offset, uint64_t file_bytes) {
    TensorInfo t;
    t.name = c.text("tensor name");
    const auto code = c.scalar<uint8_t>("tensor dtype");
    t.dtype = static_cast<DType>(code);
    if (code > static_cast<uint8_t>(DType::U8))
        fail(file + ": tensor '" + t.name + "' has dtype code " + std::to_string(code) + ", which version 1 does not define", NAVI_E_FORMAT);
    t.dims.resize(c.scalar<uint8_t>("tensor rank"));
    for (auto & d : t.dims) d = c.scalar<uint64_t>("tensor dimension");
    t.offset = c.scalar<uint64_t>("tensor offset");
    t.nbytes = c.scalar<uint64_t>("tensor byte length");
    const uint64_t room = file_bytes - data_offset;
    if (t.offset % kPage != 0) fail(file + ": tensor '" + t.name + "' starts at data byte " + std::to_string(t.offset) + ", not on a page", NAVI_E_FORMAT);
    if (t.offset > room || t.nbytes > room - t.offset)
        fail(file + ": tensor '" + t.name + "' (data bytes " + std::to_string(t.offset) + " + " + std::to_string(t.nbytes) +
                 ") runs past the end of the file",
             NAVI_E_FORMAT);
    if (t.numel() * dtype_size(t.dtype) != t.nbytes)
        fail(file + ": tensor '" + t.name + "' has " + std::to_string(t.numel()) + " elements but " + std::to_string(t.nbytes) + " bytes",
             NAVI_E_FORMAT);
    return t;
}

} // namespace

void FileUnmap::operator()(const uint8_t * p) const {
    if (p) munmap(const_cast<uint8_t *>(p), bytes);
}

NaviFile NaviFile::open(const std::string & path) {
    NaviFile f;
    f.path_ = path;
    {
        const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
        if (fd < 0) fail("cannot open " + path + ": " + std::strerror(errno), NAVI_E_FORMAT);
        struct stat st {};
        const bool sized = fstat(fd, &st) == 0;
        f.size_ = sized ? static_cast<uint64_t>(st.st_size) : 0;
        if (!sized || f.size_ < kPreambleBytes) {
            ::close(fd);
            fail(path + ": " + std::to_string(f.size_) + " bytes is shorter than a .navi preamble", NAVI_E_FORMAT);
        }
        // the upload reads every tensor front to back once
        (void) posix_fadvise(fd, 0, 0, POSIX_FADV_SEQUENTIAL);
        void * m = mmap(nullptr, f.size_, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);   // the mapping outlives the descriptor
        if (m == MAP_FAILED) fail("cannot map " + path + ": " + std::strerror(errno), NAVI_E_FORMAT);
        f.map_ = std::unique_ptr<const uint8_t, FileUnmap>(static_cast<const uint8_t *>(m), FileUnmap{f.size_});
    }
    HeaderCursor c(f.map_.get(), kPreambleBytes, path);
    const auto magic = c.scalar<uint32_t>("magic");
    const auto version = c.scalar<uint32_t>("format version");
    f.data_offset_ = c.scalar<uint64_t>("data offset");
    const auto n_kv = c.scalar<uint32_t>("hyperparameter count");
    const auto n_tensors = c.scalar<uint32_t>("tensor count");
    const auto declared = c.scalar<uint64_t>("file size");
    if (std::memcmp(&magic, "NAVI", 4) != 0) fail(path + ": the first four bytes are not 'NAVI'", NAVI_E_FORMAT);
    if (version != kFormatVersion)
        fail(path + ": format version " + std::to_string(version) + " is not supported (only version " + std::to_string(kFormatVersion) + ")",
             NAVI_E_FORMAT);
    if (declared != f.size_)
        fail(path + ": the preamble records " + std::to_string(declared) + " bytes but the file holds " + std::to_string(f.size_) +
                 " (truncated or appended to)",
             NAVI_E_FORMAT);
    if (f.data_offset_ % kPage != 0 || f.data_offset_ < kPreambleBytes || f.data_offset_ > f.size_)
        fail(path + ": data offset " + std::to_string(f.data_offset_) + " is not a page boundary inside the file", NAVI_E_FORMAT);
    c.limit(f.data_offset_);
    for (uint32_t i = 0; i < n_kv; ++i) {
        std::string key = c.text("hyperparameter key");
        KV v = decode_value(c, path, key);
        f.kv_.insert_or_assign(std::move(key), std::move(v));
    }
    f.tensors_.reserve(n_tensors);
    for (uint32_t i = 0; i < n_tensors; ++i) {
        TensorInfo t = decode_tensor(c, path, f.data_offset_, f.size_);
        const auto [it, fresh] = f.index_.try_emplace(t.name, f.tensors_.size());
        if (!fresh) fail(path + ": tensor '" + t.name + "' appears twice in the tensor table", NAVI_E_FORMAT);
        f.tensors_.push_back(std::move(t));
    }
    return f;
}

void NaviFile::close() { map_.reset(); }

bool NaviFile::has_kv(std::string_view k) const { return kv_.count(std::string(k)) != 0; }
static const KV & kv_at(const std::map<std::string, KV> & m, std::string_view k, const std::string & path) {
    const auto it = m.find(std::string(k));
    if (it == m.end()) fail(path + ": missing key '" + std::string(k) + "'", NAVI_E_FORMAT);
    return it->second;
}
int64_t NaviFile::kv_i64(std::string_view k) const {
    const KV & v = kv_at(kv_, k, path_);
    if (v.type != KV::Type::I64) fail(path_ + ": key '" + std::string(k) + "' is not an integer", NAVI_E_FORMAT);
    return v.i64;
}
int64_t NaviFile::kv_i64_or(std::string_view k, int64_t d) const { return has_kv(k) ? kv_i64(k) : d; }
double NaviFile::kv_f64(std::string_view k) const {
    const KV & v = kv_at(kv_, k, path_);
    if (v.type == KV::Type::F64) return v.f64;
    if (v.type == KV::Type::I64) return static_cast<double>(v.i64);
    fail(path_ + ": key '" + std::string(k) + "' is not a number", NAVI_E_FORMAT);
}
double NaviFile::kv_f64_or(std::string_view k, double d) const { return has_kv(k) ? kv_f64(k) : d; }
std::string NaviFile::kv_str(std::string_view k) const {
    const KV & v = kv_at(kv_, k, path_);
    if (v.type != KV::Type::STR) fail(path_ + ": key '" + std::string(k) + "' is not a string", NAVI_E_FORMAT);
    return v.str;
}
std::vector<int64_t> NaviFile::kv_i64_array(std::string_view k) const {
    const KV & v = kv_at(kv_, k, path_);
    if (v.type != KV::Type::I64_ARRAY) fail(path_ + ": key '" + std::string(k) + "' is not an integer array", NAVI_E_FORMAT);
    return v.arr;
}
const TensorInfo * NaviFile::find(std::string_view name) const {
    const auto it = index_.find(std::string(name));
    return it == index_.end() ? nullptr : &tensors_[it->second];
}
const void * NaviFile::data(const TensorInfo & t) const {
    if (!map_) fail(path_ + ": the mapping was released by close()", NAVI_E_FORMAT);
    return map_.get() + data_offset_ + t.offset;
}

// ---- parameters ---------------------------------------------------------------------------------------

static TransformerParams read_transformer(const NaviFile & f, const std::string & ns) {
    TransformerParams t;
    t.hidden = static_cast<int>(f.kv_i64(ns + ".hidden_size"));
    t.n_layer = static_cast<int>(f.kv_i64(ns + ".num_hidden_layers"));
    t.n_head = static_cast<int>(f.kv_i64(ns + ".num_attention_heads"));
    t.n_kv_head = static_cast<int>(f.kv_i64(ns + ".num_key_value_heads"));
    t.head_dim = static_cast<int>(f.kv_i64(ns + ".head_dim"));
    t.ff = static_cast<int>(f.kv_i64(ns + ".intermediate_size"));
    t.rms_eps = static_cast<float>(f.kv_f64(ns + ".rms_norm_eps"));
    t.rope_theta = f.kv_f64(ns + ".rope_theta");
    t.vocab = static_cast<int>(f.kv_i64_or(ns + ".vocab_size", 0));
    t.max_pos = static_cast<int>(f.kv_i64_or(ns + ".max_position_embeddings", 0));
    return t;
}

static std::vector<int> ints(const std::vector<int64_t> & v) { return std::vector<int>(v.begin(), v.end()); }

Params read_params(const NaviFile & f) {
    if (f.kv_str("general.arch") != "qwen3-tts") fail(f.path() + ": architecture is not qwen3-tts", NAVI_E_FORMAT);
    Params p;
    p.name = f.kv_str("general.name");
    p.im_start_id = static_cast<int>(f.kv_i64("text.im_start_id"));
    p.im_end_id = static_cast<int>(f.kv_i64("text.im_end_id"));
    p.assistant_id = static_cast<int>(f.kv_i64("text.assistant_id"));
    p.tts_bos_id = static_cast<int>(f.kv_i64("text.tts_bos_id"));
    p.tts_eos_id = static_cast<int>(f.kv_i64("text.tts_eos_id"));
    p.tts_pad_id = static_cast<int>(f.kv_i64("text.tts_pad_id"));
    p.text_vocab = static_cast<int>(f.kv_i64("talker.text_vocab_size"));
    p.text_hidden = static_cast<int>(f.kv_i64("talker.text_hidden_size"));
    p.talker = read_transformer(f, "talker");
    p.n_code_groups = static_cast<int>(f.kv_i64("talker.num_code_groups"));
    p.codec_bos_id = static_cast<int>(f.kv_i64("talker.codec_bos_id"));
    p.codec_eos_id = static_cast<int>(f.kv_i64("talker.codec_eos_token_id"));
    p.codec_pad_id = static_cast<int>(f.kv_i64("talker.codec_pad_id"));
    p.codec_think_id = static_cast<int>(f.kv_i64("talker.codec_think_id"));
    p.codec_nothink_id = static_cast<int>(f.kv_i64("talker.codec_nothink_id"));
    p.codec_think_bos_id = static_cast<int>(f.kv_i64("talker.codec_think_bos_id"));
    p.codec_think_eos_id = static_cast<int>(f.kv_i64("talker.codec_think_eos_id"));
    for (const auto & [k, v] : f.kv()) {
        const std::string pre = "talker.language.";
        if (k.compare(0, pre.size(), pre) == 0 && v.type == KV::Type::I64) p.language_ids[k.substr(pre.size())] = static_cast<int>(v.i64);
    }
    p.cp = read_transformer(f, "cp");
    p.codec_sample_rate = static_cast<int>(f.kv_i64("codec.output_sample_rate"));
    p.codec_upsample = static_cast<int>(f.kv_i64("codec.decode_upsample_rate"));
    p.vocoder = read_transformer(f, "codec.decoder");
    p.vq_latent = static_cast<int>(f.kv_i64("codec.decoder.latent_dim"));
    p.vq_codebook_dim = static_cast<int>(f.kv_i64("codec.decoder.codebook_dim"));
    p.vq_codebook_size = static_cast<int>(f.kv_i64("codec.decoder.codebook_size"));
    p.vq_n_q = static_cast<int>(f.kv_i64("codec.decoder.num_quantizers"));
    p.vq_n_semantic = static_cast<int>(f.kv_i64("codec.decoder.num_semantic_quantizers"));
    p.decoder_dim = static_cast<int>(f.kv_i64("codec.decoder.decoder_dim"));
    p.sliding_window = static_cast<int>(f.kv_i64_or("codec.decoder.sliding_window", 0));
    p.upsample_rates = ints(f.kv_i64_array("codec.decoder.upsample_rates"));
    p.upsampling_ratios = ints(f.kv_i64_array("codec.decoder.upsampling_ratios"));
    p.temperature = static_cast<float>(f.kv_f64_or("gen.temperature", 1.0));
    p.top_p = static_cast<float>(f.kv_f64_or("gen.top_p", 1.0));
    p.top_k = static_cast<int>(f.kv_i64_or("gen.top_k", 0));
    p.repetition_penalty = static_cast<float>(f.kv_f64_or("gen.repetition_penalty", 1.0));
    p.cp_temperature = static_cast<float>(f.kv_f64_or("gen.subtalker_temperature", 1.0));
    p.cp_top_p = static_cast<float>(f.kv_f64_or("gen.subtalker_top_p", 1.0));
    p.cp_top_k = static_cast<int>(f.kv_i64_or("gen.subtalker_top_k", 0));
    if (p.n_code_groups < 2) fail(f.path() + ": num_code_groups must be >= 2", NAVI_E_FORMAT);
    return p;
}

static void decoder_layers(std::vector<ExpectedTensor> & out, const std::string & prefix, const TransformerParams & t, bool qk_norm) {
    const auto H = static_cast<uint64_t>(t.hidden), Q = static_cast<uint64_t>(t.n_head * t.head_dim),
               K = static_cast<uint64_t>(t.n_kv_head * t.head_dim), F = static_cast<uint64_t>(t.ff), D = static_cast<uint64_t>(t.head_dim);
    for (int l = 0; l < t.n_layer; ++l) {
        const std::string p = prefix + ".layers." + std::to_string(l) + ".";
        out.push_back({p + "input_layernorm.weight", {H}});
        out.push_back({p + "post_attention_layernorm.weight", {H}});
        out.push_back({p + "self_attn.q_proj.weight", {Q, H}});
        out.push_back({p + "self_attn.k_proj.weight", {K, H}});
        out.push_back({p + "self_attn.v_proj.weight", {K, H}});
        out.push_back({p + "self_attn.o_proj.weight", {H, Q}});
        if (qk_norm) {
            out.push_back({p + "self_attn.q_norm.weight", {D}});
            out.push_back({p + "self_attn.k_norm.weight", {D}});
        }
        out.push_back({p + "mlp.gate_proj.weight", {F, H}});
        out.push_back({p + "mlp.up_proj.weight", {F, H}});
        out.push_back({p + "mlp.down_proj.weight", {H, F}});
    }
}

std::vector<ExpectedTensor> expected_tensors(const Params & p) {
    std::vector<ExpectedTensor> out;
    using u = uint64_t;
    const u H = p.talker.hidden, TH = p.text_hidden, TV = p.text_vocab, CV = p.talker.vocab, PV = p.cp.vocab, G = p.n_code_groups;
    out.push_back({"talker.model.text_embedding.weight", {TV, TH}});
    out.push_back({"talker.text_projection.linear_fc1.weight", {TH, TH}});
    out.push_back({"talker.text_projection.linear_fc1.bias", {TH}});
    out.push_back({"talker.text_projection.linear_fc2.weight", {H, TH}});
    out.push_back({"talker.text_projection.linear_fc2.bias", {H}});
    out.push_back({"talker.model.codec_embedding.weight", {CV, H}});
    decoder_layers(out, "talker.model", p.talker, true);
    out.push_back({"talker.model.norm.weight", {H}});
    out.push_back({"talker.codec_head.weight", {CV, H}});
    const u CH = p.cp.hidden;
    for (u i = 0; i + 1 < G; ++i) {
        out.push_back({"talker.code_predictor.model.codec_embedding." + std::to_string(i) + ".weight", {PV, CH}});
        out.push_back({"talker.code_predictor.lm_head." + std::to_string(i) + ".weight", {PV, CH}});
    }
    decoder_layers(out, "talker.code_predictor.model", p.cp, true);
    out.push_back({"talker.code_predictor.model.norm.weight", {CH}});
    // codec decoder
    const u L = p.vq_latent, CD = p.vq_codebook_dim, VQ = CD / 2, CS = p.vq_codebook_size, NQ = p.vq_n_q, NS = p.vq_n_semantic,
            DD = p.decoder_dim;
    const std::string q = "codec.decoder.quantizer.";
    out.push_back({q + "rvq_first.output_proj.weight", {CD, VQ, 1}});
    for (u i = 0; i < NS; ++i) out.push_back({q + "rvq_first.vq.layers." + std::to_string(i) + "._codebook.codebook", {CS, VQ}});
    out.push_back({q + "rvq_rest.output_proj.weight", {CD, VQ, 1}});
    for (u i = 0; i < NQ - NS; ++i) out.push_back({q + "rvq_rest.vq.layers." + std::to_string(i) + "._codebook.codebook", {CS, VQ}});
    out.push_back({"codec.decoder.pre_conv.conv.weight", {L, CD, 3}});
    out.push_back({"codec.decoder.pre_conv.conv.bias", {L}});
    const u VH = p.vocoder.hidden;
    const std::string pt = "codec.decoder.pre_transformer.";
    out.push_back({pt + "input_proj.weight", {VH, L}});
    out.push_back({pt + "input_proj.bias", {VH}});
    decoder_layers(out, "codec.decoder.pre_transformer", p.vocoder, false);
    for (int l = 0; l < p.vocoder.n_layer; ++l) {
        const std::string lp = pt + "layers." + std::to_string(l) + ".";
        out.push_back({lp + "self_attn_layer_scale.scale", {VH}});
        out.push_back({lp + "mlp_layer_scale.scale", {VH}});
    }
    out.push_back({pt + "norm.weight", {VH}});
    out.push_back({pt + "output_proj.weight", {L, VH}});
    out.push_back({pt + "output_proj.bias", {L}});
    for (size_t j = 0; j < p.upsampling_ratios.size(); ++j) {
        const u r = p.upsampling_ratios[j];
        const std::string up = "codec.decoder.upsample." + std::to_string(j) + ".";
        out.push_back({up + "0.conv.weight", {L, L, r}});
        out.push_back({up + "0.conv.bias", {L}});
        out.push_back({up + "1.dwconv.conv.weight", {L, 1, 7}});
        out.push_back({up + "1.dwconv.conv.bias", {L}});
        out.push_back({up + "1.norm.weight", {L}});
        out.push_back({up + "1.norm.bias", {L}});
        out.push_back({up + "1.pwconv1.weight", {4 * L, L}});
        out.push_back({up + "1.pwconv1.bias", {4 * L}});
        out.push_back({up + "1.pwconv2.weight", {L, 4 * L}});
        out.push_back({up + "1.pwconv2.bias", {L}});
        out.push_back({up + "1.gamma", {L}});
    }
    out.push_back({"codec.decoder.decoder.0.conv.weight", {DD, L, 7}});
    out.push_back({"codec.decoder.decoder.0.conv.bias", {DD}});
    u width = DD;
    for (size_t i = 0; i < p.upsample_rates.size(); ++i) {
        const u rate = p.upsample_rates[i], ow = width / 2;
        const std::string bp = "codec.decoder.decoder." + std::to_string(i + 1) + ".block.";
        out.push_back({bp + "0.alpha", {width}});
        out.push_back({bp + "0.beta", {width}});
        out.push_back({bp + "1.conv.weight", {width, ow, 2 * rate}});
        out.push_back({bp + "1.conv.bias", {ow}});
        for (int r = 0; r < 3; ++r) {
            const std::string rp = bp + std::to_string(2 + r) + ".";
            out.push_back({rp + "act1.alpha", {ow}});
            out.push_back({rp + "act1.beta", {ow}});
            out.push_back({rp + "conv1.conv.weight", {ow, ow, 7}});
            out.push_back({rp + "conv1.conv.bias", {ow}});
            out.push_back({rp + "act2.alpha", {ow}});
            out.push_back({rp + "act2.beta", {ow}});
            out.push_back({rp + "conv2.conv.weight", {ow, ow, 1}});
            out.push_back({rp + "conv2.conv.bias", {ow}});
        }
        width = ow;
    }
    const size_t n = p.upsample_rates.size();
    out.push_back({"codec.decoder.decoder." + std::to_string(n + 1) + ".alpha", {width}});
    out.push_back({"codec.decoder.decoder." + std::to_string(n + 1) + ".beta", {width}});
    out.push_back({"codec.decoder.decoder." + std::to_string(n + 2) + ".conv.weight", {1, width, 7}});
    out.push_back({"codec.decoder.decoder." + std::to_string(n + 2) + ".conv.bias", {1}});
    return out;
}

Validation validate(const NaviFile & f, const Params & p) {
    // expected name -> dims; each file tensor is checked against it and crossed off, and
    // whatever is left over afterwards is missing
    std::map<std::string, std::vector<uint64_t>> want;
    for (ExpectedTensor & e : expected_tensors(p)) want.emplace(std::move(e.name), std::move(e.dims));
    Validation v;
    std::set<std::string> matched;
    for (const TensorInfo & t : f.tensors()) {
        const auto it = want.find(t.name);
        if (it == want.end()) {
            v.unused.push_back(t.name);
            continue;
        }
        matched.insert(t.name);
        if (it->second != t.dims) v.shape_mismatch.push_back(t.name);
    }
    for (const auto & [name, dims] : want)
        if (!matched.count(name)) v.missing.push_back(name);
    return v;
}

// ---- device ---------------------------------------------------------------------------------------------

Device::Device(int ordinal) {
    int n = 0;
    NAVI_CUDA(cudaGetDeviceCount(&n));
    if (ordinal < 0 || ordinal >= n) fail("no CUDA device " + std::to_string(ordinal) + " (" + std::to_string(n) + " visible)", NAVI_E_ARG);
    cudaDeviceProp prop{};
    NAVI_CUDA(cudaGetDeviceProperties(&prop, ordinal));
    info_.ordinal = ordinal;
    info_.name = prop.name;
    info_.cc_major = prop.major;
    info_.cc_minor = prop.minor;
    info_.multiprocessors = prop.multiProcessorCount;
    info_.cooperative_launch = prop.cooperativeLaunch != 0;
    info_.smem_optin = prop.sharedMemPerBlockOptin;
    info_.l2_bytes = static_cast<size_t>(prop.l2CacheSize);
    if (prop.major != 10 || prop.minor != 0)
        fail("device " + std::to_string(ordinal) + " (" + info_.name + ", sm_" + std::to_string(prop.major) + std::to_string(prop.minor) +
                 ") is not sm_100: this build carries sm_100a code only", NAVI_E_ARG);
    if (!info_.cooperative_launch) fail("device " + std::to_string(ordinal) + " does not support cooperative launch", NAVI_E_ARG);
    NAVI_CUDA(cudaSetDevice(ordinal));
    // spin on completion: one launch and one wait per frame
    const cudaError_t fe = cudaSetDeviceFlags(cudaDeviceScheduleSpin);
    if (fe != cudaSuccess && fe != cudaErrorSetOnActiveProcess) cuda_check(fe, "cudaSetDeviceFlags", __FILE__, __LINE__);
    (void) cudaGetLastError();
    NAVI_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    NAVI_CUDA(cudaMemGetInfo(&info_.vram_free, &info_.vram_total));
}

Device::~Device() {
    if (stream_) {
        cudaSetDevice(info_.ordinal);
        cudaStreamDestroy(stream_);
    }
}

void Device::make_current() const { NAVI_CUDA(cudaSetDevice(info_.ordinal)); }

// ---- weights arena ---------------------------------------------------------------------------------------------

static constexpr uint64_t ALIGN = 256;
static uint64_t align_up(uint64_t n) { return (n + ALIGN - 1) / ALIGN * ALIGN; }

DeviceWeights * DeviceWeights::upload(const Device & dev, const NaviFile & f, const Groups & groups) {
    dev.make_current();
    std::map<std::string, size_t> group_of;
    for (size_t g = 0; g < groups.size(); ++g)
        for (const auto & n : groups[g]) group_of.emplace(n, g);
    std::vector<const TensorInfo *> order;
    std::vector<bool> done(groups.size(), false);
    for (const TensorInfo & t : f.tensors()) {
        if (t.dtype == DType::U8) continue;
        const auto g = group_of.find(t.name);
        if (g == group_of.end()) { order.push_back(&t); continue; }
        if (done[g->second]) continue;
        done[g->second] = true;
        for (const auto & n : groups[g->second])
            if (const TensorInfo * m = f.find(n)) order.push_back(m);
    }
    uint64_t arena = 0;
    for (const TensorInfo * t : order) arena += align_up(t->nbytes);
    auto * w = new DeviceWeights();
    w->ordinal_ = dev.info().ordinal;
    if (arena == 0) return w;
    const cudaError_t e = cudaMalloc(&w->arena_, arena);
    if (e != cudaSuccess) {
        delete w;
        fail("cannot allocate " + std::to_string(arena >> 20) + " MiB for weights: " + cudaGetErrorString(e), NAVI_E_NOMEM);
    }
    // upload through a pinned staging buffer so the copies run at PCIe speed
    const size_t STAGE = 64ull << 20;
    void * stage = nullptr;
    NAVI_CUDA(cudaMallocHost(&stage, STAGE));
    uint64_t off = 0;
    for (const TensorInfo * t : order) {
        DeviceTensor d;
        d.info = *t;
        d.ptr = static_cast<uint8_t *>(w->arena_) + off;
        const uint8_t * src = static_cast<const uint8_t *>(f.data(*t));
        for (uint64_t o = 0; o < t->nbytes; o += STAGE) {
            const size_t n = static_cast<size_t>(std::min<uint64_t>(STAGE, t->nbytes - o));
            std::memcpy(stage, src + o, n);
            NAVI_CUDA(cudaMemcpy(static_cast<uint8_t *>(d.ptr) + o, stage, n, cudaMemcpyHostToDevice));
        }
        w->tensors_.emplace(t->name, std::move(d));
        off += align_up(t->nbytes);
    }
    NAVI_CUDA(cudaFreeHost(stage));
    w->bytes_ = arena;
    return w;
}

DeviceWeights::~DeviceWeights() {
    if (arena_) {
        cudaSetDevice(ordinal_);
        cudaFree(arena_);
    }
}

const DeviceTensor * DeviceWeights::find(std::string_view name) const {
    const auto it = tensors_.find(std::string(name));
    return it == tensors_.end() ? nullptr : &it->second;
}
const DeviceTensor & DeviceWeights::get(std::string_view name) const {
    const DeviceTensor * t = find(name);
    if (!t) fail("weights: missing tensor '" + std::string(name) + "'", NAVI_E_FORMAT);
    return *t;
}

DeviceWeights::Groups fused_groups(const Params & p) {
    DeviceWeights::Groups g;
    auto add = [&](const std::string & prefix, int n_layer) {
        for (int l = 0; l < n_layer; ++l) {
            const std::string lp = prefix + ".layers." + std::to_string(l) + ".";
            g.push_back({lp + "self_attn.q_proj.weight", lp + "self_attn.k_proj.weight", lp + "self_attn.v_proj.weight"});
            g.push_back({lp + "mlp.gate_proj.weight", lp + "mlp.up_proj.weight"});
        }
    };
    add("talker.model", p.talker.n_layer);
    add("talker.code_predictor.model", p.cp.n_layer);
    return g;
}

} // namespace navi
