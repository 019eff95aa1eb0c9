// extern "C" entry points of include/navi_b200.h over the C++ classes.
#include "../../include/navi_b200.h"

#include "frame.hpp"
#include "runtime.hpp"
#include "sample_static.hpp"
#include "talker.hpp"
#include "graph.hpp"
#include "vocoder.hpp"
#include "conv_api.hpp"

#include <algorithm>
#include <cstring>
#include <memory>
#include <string>

struct navi_device {
    std::unique_ptr<navi::Device> dev;
};
struct navi_weights {
    navi::DeviceWeights * w = nullptr;
    int ordinal = 0;
};
struct navi_frame {
    std::unique_ptr<navi::qwen3tts::Frame> f;
    navi_device * dev = nullptr;
};
struct navi_talker {
    std::unique_ptr<navi::qwen3tts::Talker> t;
    int hidden = 0;
};
struct navi_graph {
    std::unique_ptr<navi::qwen3tts::Graph> g;
    int hidden = 0;
};
struct navi_vocoder {
    std::unique_ptr<navi::qwen3tts::Vocoder> v;
    int n_q = 0;
};

namespace {

thread_local std::string g_err;

int set_err(int st, const std::string & m) {
    g_err = m;
    return st;
}

template <class F> int guard(F && fn) {
    try {
        return fn();
    } catch (const navi::Error & e) {
        return set_err(e.status ? e.status : NAVI_E_ARG, e.what());
    } catch (const std::exception & e) {
        return set_err(NAVI_E_ARG, e.what());
    }
}

navi::qwen3tts::Sampling to_sampling(const navi_sampling * s) {
    navi::qwen3tts::Sampling o;
    if (!s) return o;
    o.temperature = s->temperature; o.top_k = s->top_k; o.top_p = s->top_p; o.repetition_penalty = s->repetition_penalty;
    o.cp_temperature = s->cp_temperature; o.cp_top_k = s->cp_top_k; o.cp_top_p = s->cp_top_p; o.min_frames = s->min_frames;
    o.rng = s->rng;
    return o;
}

void to_result(const navi::qwen3tts::FrameResult & r, navi_frame_result * out) {
    if (!out) return;
    std::memset(out, 0, sizeof(*out));
    out->ok = r.ok ? 1 : 0;
    out->eos = r.eos ? 1 : 0;
    std::memcpy(out->codes, r.codes, sizeof(out->codes));
    out->us = r.us;
    out->status = r.ok ? NAVI_OK : r.status;
}

void fill_params(navi_params & out, const navi::Params & p);

void fill_tp(navi_transformer_params & d, const navi::TransformerParams & s) {
    d.hidden = s.hidden; d.n_layer = s.n_layer; d.n_head = s.n_head; d.n_kv_head = s.n_kv_head; d.head_dim = s.head_dim;
    d.ff = s.ff; d.vocab = s.vocab; d.max_pos = s.max_pos; d.rms_eps = s.rms_eps; d.rope_theta = s.rope_theta;
}

} // namespace

extern "C" {

const char * navi_version(void) { return "navi-b200 0.1 (sm_100a)"; }
const char * navi_last_error(void) { return g_err.c_str(); }

int navi_device_count(int * n) {
    return guard([&]() -> int {
        if (!n) return set_err(NAVI_E_ARG, "n is NULL");
        const cudaError_t e = cudaGetDeviceCount(n);
        if (e == cudaErrorNoDevice) { *n = 0; (void) cudaGetLastError(); return NAVI_OK; }
        NAVI_CUDA(e);
        return NAVI_OK;
    });
}

int navi_device_open(int ordinal, navi_device ** out) {
    return guard([&]() -> int {
        if (!out) return set_err(NAVI_E_ARG, "out is NULL");
        auto d = std::make_unique<navi_device>();
        d->dev = std::make_unique<navi::Device>(ordinal);
        *out = d.release();
        return NAVI_OK;
    });
}

int navi_device_get_info(const navi_device * dev, navi_device_info * info) {
    return guard([&]() -> int {
        if (!dev || !info) return set_err(NAVI_E_ARG, "NULL argument");
        const auto & i = dev->dev->info();
        std::memset(info, 0, sizeof(*info));
        info->ordinal = i.ordinal;
        std::strncpy(info->name, i.name.c_str(), sizeof(info->name) - 1);
        info->cc_major = i.cc_major;
        info->cc_minor = i.cc_minor;
        info->multiprocessors = i.multiprocessors;
        info->cooperative_launch = i.cooperative_launch;
        info->smem_per_block_optin = i.smem_optin;
        info->l2_bytes = i.l2_bytes;
        info->vram_total = i.vram_total;
        info->vram_free = i.vram_free;
        return NAVI_OK;
    });
}

void * navi_device_stream(const navi_device * dev) { return dev ? static_cast<void *>(dev->dev->stream()) : nullptr; }

void navi_device_close(navi_device * dev) { delete dev; }

int navi_weights_upload(navi_device * dev, const char * path, navi_weights ** out) {
    return guard([&]() -> int {
        if (!dev || !path || !out) return set_err(NAVI_E_ARG, "NULL argument");
        navi::NaviFile f = navi::NaviFile::open(path);
        navi::Params p = navi::read_params(f);
        const navi::Validation v = navi::validate(f, p);
        if (!v.ok()) {
            std::string m = std::string(path) + ": tensor table does not match the model";
            if (!v.missing.empty()) m += " (missing " + v.missing[0] + ")";
            else m += " (shape mismatch " + v.shape_mismatch[0] + ")";
            return set_err(NAVI_E_FORMAT, m);
        }
        auto w = std::make_unique<navi_weights>();
        w->w = navi::DeviceWeights::upload(*dev->dev, f, navi::fused_groups(p));
        w->w->params_ = p;
        w->ordinal = dev->dev->info().ordinal;
        *out = w.release();
        return NAVI_OK;
    });
}

int navi_weights_get_params(const navi_weights * w, navi_params * o) {
    return guard([&]() -> int {
        if (!w || !o) return set_err(NAVI_E_ARG, "NULL argument");
        fill_params(*o, w->w->params());
        return NAVI_OK;
    });
}

int navi_model_probe(const char * path, navi_params * o, int * n_tensors, int * n_missing, int * n_mismatched, int * n_unused) {
    return guard([&]() -> int {
        if (!path) return set_err(NAVI_E_ARG, "path is NULL");
        navi::NaviFile f = navi::NaviFile::open(path);
        const navi::Params p = navi::read_params(f);
        const navi::Validation v = navi::validate(f, p);
        if (o) fill_params(*o, p);
        if (n_tensors) *n_tensors = static_cast<int>(f.tensors().size());
        if (n_missing) *n_missing = static_cast<int>(v.missing.size());
        if (n_mismatched) *n_mismatched = static_cast<int>(v.shape_mismatch.size());
        if (n_unused) *n_unused = static_cast<int>(v.unused.size());
        if (!v.missing.empty()) return set_err(NAVI_E_FORMAT, std::string(path) + ": tensor '" + v.missing[0] + "' is missing");
        if (!v.shape_mismatch.empty())
            return set_err(NAVI_E_FORMAT, std::string(path) + ": tensor '" + v.shape_mismatch[0] + "' has the wrong shape");
        return NAVI_OK;
    });
}

}   // extern "C"

namespace {
void fill_params(navi_params & out, const navi::Params & p) {
    navi_params * o = &out;
    {
        std::memset(o, 0, sizeof(*o));
        fill_tp(o->talker, p.talker);
        fill_tp(o->cp, p.cp);
        fill_tp(o->vocoder, p.vocoder);
        o->text_vocab = p.text_vocab; o->text_hidden = p.text_hidden; o->n_code_groups = p.n_code_groups;
        o->tts_bos_id = p.tts_bos_id; o->tts_eos_id = p.tts_eos_id; o->tts_pad_id = p.tts_pad_id;
        o->codec_bos_id = p.codec_bos_id; o->codec_eos_id = p.codec_eos_id; o->codec_pad_id = p.codec_pad_id;
        o->codec_think_id = p.codec_think_id; o->codec_nothink_id = p.codec_nothink_id;
        o->codec_think_bos_id = p.codec_think_bos_id; o->codec_think_eos_id = p.codec_think_eos_id;
        o->vq_latent = p.vq_latent; o->vq_codebook_dim = p.vq_codebook_dim; o->vq_codebook_size = p.vq_codebook_size;
        o->vq_n_q = p.vq_n_q; o->vq_n_semantic = p.vq_n_semantic; o->decoder_dim = p.decoder_dim; o->sliding_window = p.sliding_window;
        for (size_t i = 0; i < p.upsample_rates.size() && i < 4; ++i) o->upsample_rates[i] = p.upsample_rates[i];
        for (size_t i = 0; i < p.upsampling_ratios.size() && i < 2; ++i) o->upsampling_ratios[i] = p.upsampling_ratios[i];
        o->codec_upsample = p.codec_upsample; o->sample_rate = p.codec_sample_rate;
        o->temperature = p.temperature; o->top_p = p.top_p; o->repetition_penalty = p.repetition_penalty;
        o->cp_temperature = p.cp_temperature; o->cp_top_p = p.cp_top_p; o->top_k = p.top_k; o->cp_top_k = p.cp_top_k;
    }
}
}   // namespace

extern "C" {

const void * navi_weights_tensor(const navi_weights * w, const char * name, int * dtype, int * ndim, uint64_t dims[4]) {
    if (!w || !name) return nullptr;
    const navi::DeviceTensor * t = w->w->find(name);
    if (!t) return nullptr;
    if (dtype) *dtype = static_cast<int>(t->info.dtype);
    if (ndim) *ndim = static_cast<int>(t->info.dims.size());
    if (dims)
        for (size_t i = 0; i < 4; ++i) dims[i] = i < t->info.dims.size() ? t->info.dims[i] : 0;
    return t->ptr;
}

uint64_t navi_weights_bytes(const navi_weights * w) { return w ? w->w->bytes() : 0; }

void navi_weights_free(navi_weights * w) {
    if (!w) return;
    delete w->w;
    delete w;
}

int navi_kv_create(navi_device * dev, int n_layer, int max_pos, int kv_dim, navi_kv ** out) {
    return guard([&]() -> int {
        if (!dev || !out || n_layer <= 0 || max_pos <= 0 || kv_dim <= 0) return set_err(NAVI_E_ARG, "bad KV shape");
        dev->dev->make_current();
        auto kv = std::make_unique<navi_kv>();
        kv->n_layer = n_layer; kv->max_pos = max_pos; kv->kv_dim = kv_dim; kv->n_used = 0;
        kv->k = new uint16_t *[n_layer]();
        kv->v = new uint16_t *[n_layer]();
        const size_t bytes = static_cast<size_t>(max_pos) * kv_dim * 2;
        for (int l = 0; l < n_layer; ++l) {
            NAVI_CUDA(cudaMalloc(reinterpret_cast<void **>(&kv->k[l]), bytes));
            NAVI_CUDA(cudaMalloc(reinterpret_cast<void **>(&kv->v[l]), bytes));
            NAVI_CUDA(cudaMemset(kv->k[l], 0, bytes));
            NAVI_CUDA(cudaMemset(kv->v[l], 0, bytes));
        }
        *out = kv.release();
        return NAVI_OK;
    });
}

void navi_kv_destroy(navi_kv * kv) {
    if (!kv) return;
    for (int l = 0; l < kv->n_layer; ++l) {
        if (kv->k) cudaFree(kv->k[l]);
        if (kv->v) cudaFree(kv->v[l]);
    }
    delete[] kv->k;
    delete[] kv->v;
    delete kv;
}

int navi_frame_create(navi_device * dev, const navi_weights * w, const navi_frame_opts * opts, navi_frame ** out) {
    return guard([&]() -> int {
        if (!dev || !w || !out) return set_err(NAVI_E_ARG, "NULL argument");
        navi::qwen3tts::FrameOptions o;
        if (opts) {
            o.blocks_per_mp = opts->blocks_per_mp > 0 ? opts->blocks_per_mp : 1;
            o.deadline_us = opts->deadline_us;
        }
        auto f = std::make_unique<navi_frame>();
        f->f = navi::qwen3tts::Frame::create(*dev->dev, *w->w, o);
        f->dev = dev;
        *out = f.release();
        return NAVI_OK;
    });
}

int navi_frame_reset(navi_frame * f) {
    return guard([&]() -> int {
        if (!f) return set_err(NAVI_E_ARG, "NULL frame");
        f->f->reset();
        return NAVI_OK;
    });
}

static navi::qwen3tts::KvCache as_kv(navi_kv * kv) {
    navi::qwen3tts::KvCache k;
    k.n_layer = kv->n_layer; k.max_pos = kv->max_pos; k.kv_dim = kv->kv_dim; k.k = kv->k; k.v = kv->v; k.n_used = kv->n_used;
    return k;
}

int navi_frame_run_first(navi_frame * f, const float * d_hidden, const float * d_logits, const float * d_trailing,
                         const navi_sampling * s, uint64_t seed, int frame_index, navi_frame_result * r) {
    return guard([&]() -> int {
        if (!f || !d_hidden || !d_logits || !d_trailing) return set_err(NAVI_E_ARG, "NULL argument");
        const auto res = f->f->run_first(d_hidden, d_logits, d_trailing, to_sampling(s), seed, frame_index);
        to_result(res, r);
        return res.ok ? NAVI_OK : set_err(res.status, res.error);
    });
}

int navi_frame_run(navi_frame * f, navi_kv * kv, int n_past, const float * d_trailing, const navi_sampling * s, uint64_t seed,
                   int frame_index, navi_frame_result * r) {
    return guard([&]() -> int {
        if (!f || !kv || !d_trailing) return set_err(NAVI_E_ARG, "NULL argument");
        auto k = as_kv(kv);
        const auto res = f->f->run(k, n_past, d_trailing, to_sampling(s), seed, frame_index);
        kv->n_used = k.n_used;
        to_result(res, r);
        return res.ok ? NAVI_OK : set_err(res.status, res.error);
    });
}

int navi_frame_run_layer(navi_frame * f, int layer, const float * d_x, navi_kv * kv, int n_past, float * d_out, navi_frame_result * r) {
    return guard([&]() -> int {
        if (!f || !kv || !d_x || !d_out) return set_err(NAVI_E_ARG, "NULL argument");
        auto k = as_kv(kv);
        const auto res = f->f->run_layer(layer, d_x, k, n_past, d_out);
        to_result(res, r);
        return res.ok ? NAVI_OK : set_err(res.status, res.error);
    });
}

int navi_frame_enqueue(navi_frame * f, navi_kv * kv, int n_past, const float * d_trailing, const navi_sampling * s, uint64_t seed,
                       int frame_index) {
    return guard([&]() -> int {
        if (!f || !kv || !d_trailing) return set_err(NAVI_E_ARG, "NULL argument");
        auto k = as_kv(kv);
        std::string err;
        const int st = f->f->enqueue(k, n_past, d_trailing, to_sampling(s), seed, frame_index, err);
        kv->n_used = k.n_used;
        return st == NAVI_OK ? NAVI_OK : set_err(st, err);
    });
}

int navi_frame_collect(navi_frame * f, navi_frame_result * r) {
    return guard([&]() -> int {
        if (!f) return set_err(NAVI_E_ARG, "NULL frame");
        const auto res = f->f->collect();
        to_result(res, r);
        return res.ok ? NAVI_OK : set_err(res.status, res.error);
    });
}

int navi_frame_reset_slot(navi_frame * f, int slot) {
    return guard([&]() -> int {
        if (!f) return set_err(NAVI_E_ARG, "NULL frame");
        f->f->reset(slot);
        return NAVI_OK;
    });
}

int navi_frame_run_first_slot(navi_frame * f, int slot, const float * d_hidden, const float * d_logits, const float * d_trailing,
                              const navi_sampling * s, uint64_t seed, int frame_index, navi_frame_result * r) {
    return guard([&]() -> int {
        if (!f || !d_hidden || !d_logits || !d_trailing) return set_err(NAVI_E_ARG, "NULL argument");
        const auto res = f->f->run_first(d_hidden, d_logits, d_trailing, to_sampling(s), seed, frame_index, slot);
        to_result(res, r);
        return res.ok ? NAVI_OK : set_err(res.status, res.error);
    });
}

int navi_frame_enqueue_batch(navi_frame * f, int nb, const int * slots, navi_kv * const * kvs, const int * n_past,
                             const float * const * d_trailing, const navi_sampling * s, const uint64_t * seeds, const int * frame_index) {
    return guard([&]() -> int {
        if (!f || !slots || !kvs || !n_past || !d_trailing || !seeds || !frame_index) return set_err(NAVI_E_ARG, "NULL argument");
        if (nb < 1 || nb > navi::qwen3tts::Frame::MAX_SLOTS) return set_err(NAVI_E_ARG, "stream count out of range");
        navi::qwen3tts::KvCache k[navi::qwen3tts::Frame::MAX_SLOTS];
        navi::qwen3tts::KvCache * kp[navi::qwen3tts::Frame::MAX_SLOTS];
        for (int i = 0; i < nb; ++i) {
            if (!kvs[i]) return set_err(NAVI_E_ARG, "NULL KV cache");
            k[i] = as_kv(kvs[i]);
            kp[i] = &k[i];
        }
        std::string err;
        const int st = f->f->enqueue_batch(nb, slots, kp, n_past, d_trailing, to_sampling(s), seeds, frame_index, err);
        if (st != NAVI_OK) return set_err(st, err);
        for (int i = 0; i < nb; ++i) kvs[i]->n_used = k[i].n_used;
        return NAVI_OK;
    });
}

int navi_frame_run_first_batch(navi_frame * f, int nb, const int * slots, const float * const * d_hidden, const float * const * d_logits,
                               const float * const * d_trailing, const navi_sampling * s, const uint64_t * seeds, const int * frame_index,
                               navi_frame_result * results) {
    const int st = guard([&]() -> int {
        if (!f || !slots || !d_hidden || !d_logits || !d_trailing || !seeds || !frame_index || !results) return set_err(NAVI_E_ARG, "NULL argument");
        std::string err;
        const int e = f->f->enqueue_first_batch(nb, slots, d_hidden, d_logits, d_trailing, to_sampling(s), seeds, frame_index, err);
        return e != NAVI_OK ? set_err(e, err) : NAVI_OK;
    });
    if (st != NAVI_OK) return st;
    return navi_frame_collect_batch(f, nb, results);
}
int navi_frame_collect_batch(navi_frame * f, int nb, navi_frame_result * results) {
    return guard([&]() -> int {
        if (!f || !results) return set_err(NAVI_E_ARG, "NULL argument");
        if (nb < 1 || nb > navi::qwen3tts::Frame::MAX_SLOTS) return set_err(NAVI_E_ARG, "stream count out of range");
        navi::qwen3tts::FrameResult res[navi::qwen3tts::Frame::MAX_SLOTS];
        f->f->collect_batch(res);
        int st = NAVI_OK;
        for (int i = 0; i < nb; ++i) {
            to_result(res[i], &results[i]);
            if (!res[i].ok && st == NAVI_OK) st = set_err(res[i].status, res[i].error);
        }
        return st;
    });
}

int navi_frame_run_batch(navi_frame * f, int nb, const int * slots, navi_kv * const * kvs, const int * n_past,
                         const float * const * d_trailing, const navi_sampling * s, const uint64_t * seeds, const int * frame_index,
                         navi_frame_result * results) {
    const int st = navi_frame_enqueue_batch(f, nb, slots, kvs, n_past, d_trailing, s, seeds, frame_index);
    if (st != NAVI_OK) return st;
    return navi_frame_collect_batch(f, nb, results);
}

const float * navi_frame_step_out_slot(const navi_frame * f, int slot) { return f ? f->f->d_step_out(slot) : nullptr; }

int navi_frame_set_step_in_slot(navi_frame * f, int slot, const float * d_step) {
    return guard([&]() -> int {
        if (!f || !d_step) return set_err(NAVI_E_ARG, "NULL argument");
        f->f->set_step_in(d_step, slot);
        return NAVI_OK;
    });
}

int navi_frame_inspect_stream(const navi_frame * f, int index, float * h_hidden, float * h_logits, float * h_clogits) {
    return guard([&]() -> int {
        if (!f) return set_err(NAVI_E_ARG, "NULL frame");
        f->f->inspect(h_hidden, h_logits, h_clogits, index);
        return NAVI_OK;
    });
}

const float * navi_frame_step_out(const navi_frame * f) { return f ? f->f->d_step_out() : nullptr; }

int navi_frame_set_step_in(navi_frame * f, const float * d_step) {
    return guard([&]() -> int {
        if (!f || !d_step) return set_err(NAVI_E_ARG, "NULL argument");
        f->f->set_step_in(d_step);
        return NAVI_OK;
    });
}

int navi_frame_grid_blocks(const navi_frame * f) { return f ? f->f->grid_blocks() : 0; }

void navi_frame_destroy(navi_frame * f) { delete f; }

int navi_frame_inspect(const navi_frame * f, float * h_hidden, float * h_logits, float * h_clogits) {
    return guard([&]() -> int {
        if (!f) return set_err(NAVI_E_ARG, "NULL frame");
        f->f->inspect(h_hidden, h_logits, h_clogits);
        return NAVI_OK;
    });
}

int navi_frame_set_profile(navi_frame * f, int enable, int cta) {
    return guard([&]() -> int {
        if (!f) return set_err(NAVI_E_ARG, "NULL frame");
        f->f->set_profile(enable != 0, cta);
        return NAVI_OK;
    });
}

int navi_frame_profile(const navi_frame * f, uint64_t * out, int cap, int * n) {
    return guard([&]() -> int {
        if (!f || !out || !n) return set_err(NAVI_E_ARG, "NULL argument");
        *n = f->f->profile(out, cap);
        return NAVI_OK;
    });
}

int navi_sample_logits(navi_device * dev, const float * d_logits, int vocab, const navi_sampling * s, uint64_t seed, int frame_index,
                       int codebook, int suppress_from, int eos_id, const uint8_t * d_seen, int32_t * out) {
    return guard([&]() -> int {
        if (!dev || !d_logits || !out || vocab <= 0) return set_err(NAVI_E_ARG, "bad argument");
        *out = navi::qwen3tts::Frame::sample(*dev->dev, d_logits, vocab, to_sampling(s), seed, frame_index, codebook, suppress_from,
                                             eos_id, d_seen);
        return NAVI_OK;
    });
}

int navi_sample_logits_static(navi_device * dev, const float * d_logits, int vocab, const navi_sampling * s, uint64_t seed,
                              int frame_index, int codebook, int suppress_from, int eos_id, const uint8_t * d_seen,
                              int32_t * out) {
    static_assert(NAVI_SAMPLE_STATIC_MAX_VOCAB == navi::qwen3tts::SAMPLE_STATIC_MAX_VOCAB, "limit in the header");
    return guard([&]() -> int {
        if (!dev || !d_logits || !out) return set_err(NAVI_E_ARG, "bad argument");
        *out = navi::qwen3tts::sample_static(*dev->dev, d_logits, vocab, to_sampling(s), seed, frame_index, codebook,
                                             suppress_from, eos_id, d_seen);
        return NAVI_OK;
    });
}

int navi_talker_create(navi_device * dev, const navi_weights * w, int max_prompt_tokens, int max_positions, navi_talker ** out) {
    return guard([&]() -> int {
        if (!dev || !w || !out) return set_err(NAVI_E_ARG, "NULL argument");
        auto t = std::make_unique<navi_talker>();
        t->t = navi::qwen3tts::Talker::create(*dev->dev, *w->w, max_prompt_tokens, max_positions);
        t->hidden = w->w->params().talker.hidden;
        *out = t.release();
        return NAVI_OK;
    });
}

int navi_talker_build_prompt(navi_talker * t, const int32_t * ids, int n_ids, const char * language, const float * speaker,
                             navi_prompt * out) {
    return guard([&]() -> int {
        if (!t || !ids || n_ids <= 0 || !speaker || !out) return set_err(NAVI_E_ARG, "bad argument");
        const auto & pr = t->t->build_prompt(std::span<const std::int32_t>(ids, static_cast<size_t>(n_ids)), language ? language : "",
                                             std::span<const float>(speaker, static_cast<size_t>(t->hidden)));
        out->prefill = pr.prefill;
        out->trailing = pr.trailing;
        out->tts_pad = pr.tts_pad;
        out->n_prefill = pr.n_prefill;
        out->n_trailing = pr.n_trailing;
        return NAVI_OK;
    });
}

int navi_talker_prefill(navi_talker * t, const navi_prompt * p) {
    return guard([&]() -> int {
        if (!t || !p) return set_err(NAVI_E_ARG, "NULL argument");
        navi::qwen3tts::Prompt pr;
        pr.prefill = p->prefill;
        pr.trailing = p->trailing;
        pr.tts_pad = p->tts_pad;
        pr.n_prefill = p->n_prefill;
        pr.n_trailing = p->n_trailing;
        t->t->prefill(pr);
        return NAVI_OK;
    });
}

int navi_talker_kv(navi_talker * t, navi_kv * out) {
    return guard([&]() -> int {
        if (!t || !out) return set_err(NAVI_E_ARG, "NULL argument");
        auto & kv = t->t->kv();
        out->n_layer = kv.n_layer;
        out->max_pos = kv.max_pos;
        out->kv_dim = kv.kv_dim;
        out->n_used = kv.n_used;
        out->k = kv.k;
        out->v = kv.v;
        return NAVI_OK;
    });
}

const float * navi_talker_hidden(const navi_talker * t) { return t ? t->t->d_hidden() : nullptr; }
const float * navi_talker_logits(const navi_talker * t) { return t ? t->t->d_logits() : nullptr; }
double navi_talker_last_ms(const navi_talker * t) { return t ? t->t->last_ms() : 0.0; }
void navi_talker_destroy(navi_talker * t) { delete t; }

int navi_graph_create(navi_device * dev, const navi_weights * w, const navi_frame_opts * opts, int max_prompt_tokens, int max_frames,
                      int vocoder_chunk, navi_graph ** out) {
    return guard([&]() -> int {
        if (!dev || !w || !out) return set_err(NAVI_E_ARG, "NULL argument");
        if (vocoder_chunk < 0) return set_err(NAVI_E_ARG, "vocoder_chunk must be >= 0");
        navi::qwen3tts::FrameOptions fo;
        if (opts) {
            fo.blocks_per_mp = opts->blocks_per_mp;
            if (opts->deadline_us) fo.deadline_us = opts->deadline_us;
        }
        auto g = std::make_unique<navi_graph>();
        g->g = navi::qwen3tts::Graph::create(*dev->dev, *w->w, fo, max_prompt_tokens, max_frames, vocoder_chunk);
        g->hidden = w->w->params().talker.hidden;
        *out = g.release();
        return NAVI_OK;
    });
}

namespace {

void put_stats(const navi::qwen3tts::SynthStats & s, navi_synth_stats * st) {
    if (!st) return;
    st->n_tokens = s.n_tokens;
    st->n_frames = s.n_frames;
    st->hit_cap = s.hit_cap ? 1 : 0;
    st->eos = s.eos ? 1 : 0;
    st->prefill_ms = s.prefill_ms;
    st->frames_ms = s.frames_ms;
    st->total_ms = s.total_ms;
    st->ttfc_ms = s.ttfc_ms;
    st->vocoder_ms = s.vocoder_ms;
    st->ttfa_ms = s.ttfa_ms;
    st->audio_s = s.audio_s;
    st->rtf = s.rtf;
}

navi::qwen3tts::SynthRequest make_request(const navi_graph * g, const int32_t * ids, int n_ids, const char * language,
                                          const float * speaker, const navi_sampling * s, uint64_t seed, int max_frames) {
    navi::qwen3tts::SynthRequest req;
    req.ids = std::span<const std::int32_t>(ids, static_cast<size_t>(n_ids));
    req.language = language ? language : "";
    req.speaker = std::span<const float>(speaker, static_cast<size_t>(g->hidden));
    req.seed = seed;
    req.max_frames = max_frames;
    req.sampling = to_sampling(s);
    return req;
}

} // namespace

int navi_graph_synth_ids(navi_graph * g, const int32_t * ids, int n_ids, const char * language, const float * speaker,
                         const navi_sampling * s, uint64_t seed, int max_frames, int32_t * codes, int codes_cap, navi_synth_stats * st) {
    return guard([&]() -> int {
        if (!g || !ids || n_ids <= 0 || !speaker || !codes || codes_cap <= 0) return set_err(NAVI_E_ARG, "bad argument");
        auto req = make_request(g, ids, n_ids, language, speaker, s, seed, std::min(max_frames, codes_cap));
        int n = 0;
        const auto stats = g->g->synth(req, [&](const std::int32_t * c) {
            std::memcpy(codes + static_cast<size_t>(n) * 16, c, 16 * sizeof(int32_t));
            ++n;
        });
        put_stats(stats, st);
        return NAVI_OK;
    });
}

int navi_graph_create_streams(navi_device * dev, const navi_weights * w, const navi_frame_opts * opts, int max_prompt_tokens,
                              int max_frames, int vocoder_chunk, int max_streams, navi_graph ** out) {
    return guard([&]() -> int {
        if (!dev || !w || !out) return set_err(NAVI_E_ARG, "NULL argument");
        if (vocoder_chunk < 0) return set_err(NAVI_E_ARG, "vocoder_chunk must be >= 0");
        navi::qwen3tts::FrameOptions fo;
        if (opts) {
            fo.blocks_per_mp = opts->blocks_per_mp;
            if (opts->deadline_us) fo.deadline_us = opts->deadline_us;
        }
        auto g = std::make_unique<navi_graph>();
        g->g = navi::qwen3tts::Graph::create(*dev->dev, *w->w, fo, max_prompt_tokens, max_frames, vocoder_chunk, max_streams);
        g->hidden = w->w->params().talker.hidden;
        *out = g.release();
        return NAVI_OK;
    });
}

int navi_graph_synth_batch(navi_graph * g, int n, const navi_synth_request * reqs, const navi_sampling * s, int first_batch,
                           int vocoder_batch, navi_stream_pcm_fn on_pcm, void * user, navi_synth_stats * stats) {
    return guard([&]() -> int {
        if (!g || !reqs || n < 1 || n > g->g->max_streams()) return set_err(NAVI_E_ARG, "bad argument");
        if (first_batch < 0 || vocoder_batch < 0) return set_err(NAVI_E_ARG, "batch sizes must be >= 0");
        if (on_pcm && !g->g->vocoder()) return set_err(NAVI_E_ARG, "graph created without a vocoder (vocoder_chunk = 0)");
        std::vector<navi::qwen3tts::SynthRequest> rq;
        std::vector<int> made(static_cast<size_t>(n), 0);
        for (int i = 0; i < n; ++i) {
            const navi_synth_request & r = reqs[i];
            if (!r.ids || r.n_ids <= 0 || !r.speaker || (r.codes && r.codes_cap <= 0)) return set_err(NAVI_E_ARG, "bad request");
            auto q = make_request(g, r.ids, r.n_ids, r.language, r.speaker, s, r.seed, r.codes ? std::min(r.max_frames, r.codes_cap) : r.max_frames);
            q.first_batch = first_batch;
            q.vocoder_batch = vocoder_batch;
            rq.push_back(q);
        }
        navi::qwen3tts::Graph::StreamPcmFn pcm_fn;
        if (on_pcm) pcm_fn = [&](int st, std::span<const float> pcm) { on_pcm(st, pcm.data(), static_cast<int>(pcm.size()), user); };
        const auto out = g->g->synth_batch(
            rq,
            [&](int st, const std::int32_t * c) {
                const navi_synth_request & r = reqs[st];
                int & k = made[static_cast<size_t>(st)];
                if (r.codes) std::memcpy(r.codes + static_cast<size_t>(k) * 16, c, 16 * sizeof(int32_t));
                ++k;
            },
            pcm_fn);
        if (stats)
            for (int i = 0; i < n; ++i) put_stats(out[static_cast<size_t>(i)], &stats[i]);
        return NAVI_OK;
    });
}

int navi_graph_synth(navi_graph * g, const int32_t * ids, int n_ids, const char * language, const float * speaker,
                     const navi_sampling * s, uint64_t seed, int max_frames, int first_batch, int vocoder_batch, int32_t * codes,
                     int codes_cap, navi_pcm_fn on_pcm, void * user, navi_synth_stats * st) {
    return guard([&]() -> int {
        if (!g || !ids || n_ids <= 0 || !speaker || !on_pcm || (codes && codes_cap <= 0)) return set_err(NAVI_E_ARG, "bad argument");
        if (first_batch < 0 || vocoder_batch < 0) return set_err(NAVI_E_ARG, "batch sizes must be >= 0");
        if (!g->g->vocoder()) return set_err(NAVI_E_ARG, "graph created without a vocoder (vocoder_chunk = 0)");
        auto req = make_request(g, ids, n_ids, language, speaker, s, seed, codes ? std::min(max_frames, codes_cap) : max_frames);
        req.first_batch = first_batch;
        req.vocoder_batch = vocoder_batch;
        int n = 0;
        const auto stats = g->g->synth(
            req,
            [&](const std::int32_t * c) {
                if (codes) std::memcpy(codes + static_cast<size_t>(n) * 16, c, 16 * sizeof(int32_t));
                ++n;
            },
            [&](std::span<const float> pcm) { on_pcm(pcm.data(), static_cast<int>(pcm.size()), user); });
        put_stats(stats, st);
        return NAVI_OK;
    });
}

void navi_graph_destroy(navi_graph * g) { delete g; }

int navi_vocoder_create(navi_device * dev, const navi_weights * w, int max_chunk_frames, int max_frames, navi_vocoder ** out) {
    return guard([&]() -> int {
        if (!dev || !w || !out) return set_err(NAVI_E_ARG, "NULL argument");
        auto v = std::make_unique<navi_vocoder>();
        v->v = navi::qwen3tts::Vocoder::create(*dev->dev, *w->w, max_chunk_frames, max_frames);
        v->n_q = w->w->params().vq_n_q;
        *out = v.release();
        return NAVI_OK;
    });
}

int navi_vocoder_reset(navi_vocoder * v) {
    return guard([&]() -> int {
        if (!v) return set_err(NAVI_E_ARG, "NULL argument");
        v->v->reset();
        return NAVI_OK;
    });
}

int navi_vocoder_decode(navi_vocoder * v, const int32_t * h_codes, int n_frames, float * h_pcm, size_t cap) {
    return guard([&]() -> int {
        if (!v || (n_frames > 0 && (!h_codes || !h_pcm)) || n_frames < 0) return set_err(NAVI_E_ARG, "bad argument");
        const size_t need = static_cast<size_t>(n_frames) * static_cast<size_t>(v->v->samples_per_frame());
        if (cap < need) return set_err(NAVI_E_ARG, "pcm buffer smaller than n_frames * samples_per_frame");
        v->v->decode_into(std::span<const std::int32_t>(h_codes, static_cast<size_t>(n_frames) * v->n_q), n_frames, h_pcm);
        return NAVI_OK;
    });
}

int navi_vocoder_samples_per_frame(const navi_vocoder * v) { return v ? v->v->samples_per_frame() : 0; }
int navi_vocoder_max_chunk_frames(const navi_vocoder * v) { return v ? v->v->max_chunk_frames() : 0; }
double navi_vocoder_last_ms(const navi_vocoder * v) { return v ? v->v->last_ms() : 0.0; }

int navi_vocoder_set_stage_hook(navi_vocoder * v, navi_stage_fn fn, void * user) {
    return guard([&]() -> int {
        if (!v) return set_err(NAVI_E_ARG, "NULL argument");
        if (!fn) v->v->set_stage_hook({});
        else v->v->set_stage_hook([fn, user](const char * name, const float * d, int rows, int cols) { fn(user, name, d, rows, cols); });
        return NAVI_OK;
    });
}

void navi_vocoder_destroy(navi_vocoder * v) { delete v; }

int navi_conv1d(navi_device * dev, const navi_conv_args * a) {
    return guard([&]() -> int {
        if (!dev || !a || !a->w || !a->x || !a->y) return set_err(NAVI_E_ARG, "NULL argument");
        if (a->Cout <= 0 || a->Cin <= 0 || a->K <= 0 || a->dil <= 0 || a->T < 0 || a->trans_stride < 0) return set_err(NAVI_E_ARG, "bad shape");
        if (a->trans_stride > 0 && (a->hist ? a->dil != 1 : false)) return set_err(NAVI_E_ARG, "transposed conv has dilation 1");
        return navi::conv_once(*dev->dev, *a);
    });
}

} // extern "C"
