/* navi_b200.h -- C ABI of the B200 (sm_100a) frame-decode engine.
 *
 * The reference engine (navi-tts) exposes its hot path as C++ classes; this
 * header is the flat C boundary those classes sit on here, so a C, cgo, JNI or
 * ctypes host can drive the same path.  Every entry point names the reference
 * interface it replaces.  All functions return NAVI_OK or a status code;
 * navi_last_error() gives the calling thread's message for the last failure.
 * Device pointers are plain addresses on the navi_device's GPU.  A handle is
 * used from one host thread at a time; handles on different GPUs are
 * independent (request-parallel serving pins one device per thread).
 */
#ifndef NAVI_B200_H
#define NAVI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---- status codes (reference: navi::Error thrown at setup, FrameResult{ok,error}
 *      on the request path; runtime/common/error.h:10-14, model/qwen3tts/frame.h:38-44) */
enum {
    NAVI_OK = 0,
    NAVI_E_ARG = 1,       /* bad argument */
    NAVI_E_CUDA = 2,      /* a CUDA runtime call failed */
    NAVI_E_FORMAT = 3,    /* .navi file unreadable, or its tensor table does not match the model */
    NAVI_E_TIMEOUT = 4,   /* a device-side wait passed its deadline; the frame failed, state is clean */
    NAVI_E_KV_FULL = 5,   /* n_past >= the KV cache's max_pos */
    NAVI_E_LAUNCH = 6,    /* the cooperative launch was refused */
    NAVI_E_SHAPE = 7,     /* model shape outside what the kernels are built for */
    NAVI_E_NOMEM = 8      /* device memory exhausted */
};

enum { NAVI_RNG_PCG = 0, NAVI_RNG_PHILOX = 1 };

typedef struct navi_device navi_device;
typedef struct navi_weights navi_weights;
typedef struct navi_frame navi_frame;

/* ---- library ------------------------------------------------------------------------- */

const char * navi_version(void);
/* Message of the calling thread's last failed call ("" if none). */
const char * navi_last_error(void);

/* ---- device: replaces navi::Device (runtime/device/device.h:43-66, device.cpp:77-108) --- */

typedef struct navi_device_info {
    int ordinal;
    char name[128];
    int cc_major, cc_minor;
    int multiprocessors;
    int cooperative_launch;
    size_t smem_per_block_optin;
    size_t l2_bytes;
    size_t vram_total, vram_free;
} navi_device_info;

int navi_device_count(int * n);
/* Opens GPU `ordinal` (explicit, for request-parallel pinning): requires sm_100,
 * cooperative launch; sets spin-wait scheduling; creates the engine stream. */
int navi_device_open(int ordinal, navi_device ** out);
int navi_device_get_info(const navi_device * dev, navi_device_info * info);
/* The engine's cudaStream_t. */
void * navi_device_stream(const navi_device * dev);
/* Destroy every handle made on this device (weights, KV caches, talkers, frames, vocoders,
 * graphs) first: their destroy calls use the device's stream. */
void navi_device_close(navi_device * dev);

/* ---- weights: replaces NaviFile + read_params + validate + DeviceWeights::upload
 *      (runtime/weights/navi_file.h:40-83, device_weights.h:30-61, model/qwen3tts/params.h:17-95) */

typedef struct navi_transformer_params {
    int hidden, n_layer, n_head, n_kv_head, head_dim, ff, vocab, max_pos;
    float rms_eps;
    double rope_theta;
} navi_transformer_params;

typedef struct navi_params {
    navi_transformer_params talker, cp, vocoder;
    int text_vocab, text_hidden, n_code_groups;
    int tts_bos_id, tts_eos_id, tts_pad_id;
    int codec_bos_id, codec_eos_id, codec_pad_id;
    int codec_think_id, codec_nothink_id, codec_think_bos_id, codec_think_eos_id;
    int vq_latent, vq_codebook_dim, vq_codebook_size, vq_n_q, vq_n_semantic;
    int decoder_dim, sliding_window;
    int upsample_rates[4], upsampling_ratios[2];
    int codec_upsample, sample_rate;
    float temperature, top_p, repetition_penalty, cp_temperature, cp_top_p;
    int top_k, cp_top_k;
} navi_params;

/* mmaps a .navi v1 file, validates its tensor table against the model its KV
 * section describes, and uploads every weight into one 256-byte-aligned device
 * arena (q/k/v and gate/up of each talker / code-predictor layer adjacent). */
int navi_weights_upload(navi_device * dev, const char * path, navi_weights ** out);
int navi_weights_get_params(const navi_weights * w, navi_params * p);
/* Host only (no device): reads a .navi file's header and KV section and checks its tensor
 * table against the model the KV section describes, as `navi-tts info` does without
 * --upload (runtime/cli/main.cpp:247-279 -> NaviFile::open, read_params, validate;
 * runtime/weights/navi_file.cpp:79-148, model/qwen3tts/params.cpp:59-130, 286-303).
 * p may be NULL. n_tensors / n_missing / n_mismatched / n_unused (each may be NULL) get the
 * table's counts; NAVI_E_FORMAT when the file is malformed or a tensor is missing or
 * mis-shaped, with the first such name in navi_last_error(). */
int navi_model_probe(const char * path, navi_params * p, int * n_tensors, int * n_missing, int * n_mismatched, int * n_unused);
/* Device address of a tensor by its .navi name (NULL if absent); dtype per the .navi codes. */
const void * navi_weights_tensor(const navi_weights * w, const char * name, int * dtype, int * ndim, uint64_t dims[4]);
uint64_t navi_weights_bytes(const navi_weights * w);
void navi_weights_free(navi_weights * w);

/* ---- KV cache: replaces navi::qwen3tts::KvCache (model/qwen3tts/talker.h:20-24);
 *      per layer [max_pos][kv_dim] f16, K stored after RoPE. k/v are host arrays of
 *      n_layer device pointers. */

typedef struct navi_kv {
    int n_layer, max_pos, kv_dim, n_used;
    uint16_t ** k;
    uint16_t ** v;
} navi_kv;

int navi_kv_create(navi_device * dev, int n_layer, int max_pos, int kv_dim, navi_kv ** out);
void navi_kv_destroy(navi_kv * kv);

/* ---- talker: replaces navi::qwen3tts::Talker (model/qwen3tts/talker.h:20-67) ------------- */

typedef struct navi_talker navi_talker;

typedef struct navi_prompt {        /* Prompt, talker.h:26-32: device rows, valid until the next build_prompt */
    const float * prefill;          /* [n_prefill][hidden] */
    const float * trailing;         /* [n_trailing][hidden]: frame i feeds trailing[i], then tts_pad */
    const float * tts_pad;          /* [hidden] */
    int n_prefill, n_trailing;
} navi_prompt;

/* Talker::create (talker.hip:200-266): the prompt / prefill scratch and the talker's KV
 * cache (max_positions per layer). 9 <= max_prompt_tokens <= max_positions; the prefill
 * attention has no key cap of its own. */
int navi_talker_create(navi_device * dev, const navi_weights * w, int max_prompt_tokens, int max_positions, navi_talker ** out);
/* Talker::build_prompt (talker.hip:283-352): ids = the tokenised
 * "<|im_start|>assistant\n{text}<|im_end|>\n<|im_start|>assistant\n" (3 header ids, the
 * text, 5 trailer ids); language NULL, "" or "auto" for none; speaker: host [hidden]. */
int navi_talker_build_prompt(navi_talker * t, const int32_t * ids, int n_ids, const char * language, const float * speaker,
                             navi_prompt * out);
/* Talker::prefill (talker.hip:355-399): the prefill rows at positions 0..n-1; fills the KV cache. */
int navi_talker_prefill(navi_talker * t, const navi_prompt * p);
/* Talker::kv: the talker's cache as a navi_kv (its k / v arrays belong to the talker). */
int navi_talker_kv(navi_talker * t, navi_kv * out);
/* Talker::d_hidden / d_logits: the last prefill row's post-norm hidden [hidden] and codec
 * logits [talker vocab] (the inputs of navi_frame_run_first). */
const float * navi_talker_hidden(const navi_talker * t);
const float * navi_talker_logits(const navi_talker * t);
/* Talker::last_ms: device time of the last prefill. */
double navi_talker_last_ms(const navi_talker * t);
void navi_talker_destroy(navi_talker * t);

/* ---- frame: replaces navi::qwen3tts::Frame (model/qwen3tts/frame.h:24-71) --------------- */

typedef struct navi_sampling {      /* Sampling, frame.h:24-31, plus top-p and the stream choice */
    float temperature;              /* <= 0: greedy */
    int top_k;                      /* 0 or >= vocab: off */
    float top_p;                    /* outside (0, 1): off */
    float repetition_penalty;       /* <= 0: off; over codebook-0 ids seen this request */
    float cp_temperature;
    int cp_top_k;
    float cp_top_p;
    int min_frames;                 /* EOS suppressed before this many frames */
    int rng;                        /* NAVI_RNG_PCG (the reference's stream) or NAVI_RNG_PHILOX */
} navi_sampling;

typedef struct navi_frame_opts {    /* FrameOptions, frame.h:33-36 */
    int blocks_per_mp;              /* 1 */
    uint64_t deadline_us;           /* longest any single device-side wait may take; 0: 200000 */
} navi_frame_opts;

typedef struct navi_frame_result {  /* FrameResult, frame.h:38-44 */
    int ok;
    int eos;
    int32_t codes[16];
    double us;                      /* device time of the launch */
    int status;                     /* NAVI_OK or the failure's status code */
} navi_frame_result;

/* Frame::create (frame.hip:684-774) */
int navi_frame_create(navi_device * dev, const navi_weights * w, const navi_frame_opts * opts, navi_frame ** out);
/* Frame::reset (frame.hip:783-785): clears the repetition set for a new request. */
int navi_frame_reset(navi_frame * f);
/* Frame::run_first (frame.hip:787-796): frame 0 from the prefill's post-norm hidden and logits. */
int navi_frame_run_first(navi_frame * f, const float * d_hidden, const float * d_logits, const float * d_trailing,
                         const navi_sampling * s, uint64_t seed, int frame_index, navi_frame_result * r);
/* Frame::run (frame.hip:798-810): talker step at n_past on the previous frame's step embedding. */
int navi_frame_run(navi_frame * f, navi_kv * kv, int n_past, const float * d_trailing, const navi_sampling * s,
                   uint64_t seed, int frame_index, navi_frame_result * r);
/* One talker decoder layer alone at position n_past: the layer phases of k_frame
 * (frame.hip:300-402: RMSNorm, q/k/v, q/k norm + RoPE, K/V row n_past stored, GQA
 * attention over positions 0..n_past, o + residual, RMSNorm, gate/up SwiGLU, down +
 * residual) on the f32 input d_x [hidden], the f32 output written to d_out [hidden]
 * (configs[0]'s single-layer step; the reference has no separate entry point for it).
 * r->us is the launch's device time; r->codes are not set. */
int navi_frame_run_layer(navi_frame * f, int layer, const float * d_x, navi_kv * kv, int n_past, float * d_out,
                         navi_frame_result * r);
/* Enqueue-only form of navi_frame_run (no host synchronisation, no result): for
 * pipelined loops; navi_frame_collect() then returns the last enqueued frame's result. */
int navi_frame_enqueue(navi_frame * f, navi_kv * kv, int n_past, const float * d_trailing, const navi_sampling * s,
                       uint64_t seed, int frame_index);
int navi_frame_collect(navi_frame * f, navi_frame_result * r);
/* Frame::d_step_out: the next frame's step embedding [hidden] (valid until the next run). */
const float * navi_frame_step_out(const navi_frame * f);
/* Overrides the step embedding the next navi_frame_run starts from (device [hidden]). */
int navi_frame_set_step_in(navi_frame * f, const float * d_step);
/* Frame::grid_blocks / occupancy_per_mp */
int navi_frame_grid_blocks(const navi_frame * f);

/* ---- batched decode (no counterpart in the reference, which decodes one stream per launch,
 *      the reference's docs/DESIGN.md:35; the per-stream math is Frame::run's, frame.hip:798-810) ----
 * A frame keeps NAVI_FRAME_SLOTS stream slots, each with its own repetition set and step
 * embedding; the single-stream calls above use slot 0. navi_frame_run_batch decodes one frame
 * of nb = 1, 2 or 4 streams in distinct slots in one launch that reads every weight once:
 * stream i at position n_past[i] of its own KV cache kvs[i], with its own trailing row, seed and
 * frame index; results[i] gets stream i's codes. Each stream's codes are those of
 * navi_frame_run on that stream alone, bit for bit; its hidden state and logits agree within
 * float rounding. KV length per stream is limited by the per-stream attention split
 * (NAVI_E_KV_FULL beyond it: about 1000 positions at nb = 4, 2000 at nb = 2). */
#define NAVI_FRAME_SLOTS 4
int navi_frame_reset_slot(navi_frame * f, int slot);
/* Frame 0 of the stream in `slot` (navi_frame_run_first for that slot). */
int navi_frame_run_first_slot(navi_frame * f, int slot, const float * d_hidden, const float * d_logits, const float * d_trailing,
                              const navi_sampling * s, uint64_t seed, int frame_index, navi_frame_result * r);
int navi_frame_run_batch(navi_frame * f, int nb, const int * slots, navi_kv * const * kvs, const int * n_past,
                         const float * const * d_trailing, const navi_sampling * s, const uint64_t * seeds, const int * frame_index,
                         navi_frame_result * results);
/* Frame 0 of nb = 2 or 4 streams in distinct slots in one launch: navi_frame_run_first_slot of
 * each stream together (the code predictor only), stream i from d_hidden[i] and d_logits[i] of
 * its prefill; codes bit for bit those of navi_frame_run_first_slot on that stream alone. */
int navi_frame_run_first_batch(navi_frame * f, int nb, const int * slots, const float * const * d_hidden, const float * const * d_logits,
                               const float * const * d_trailing, const navi_sampling * s, const uint64_t * seeds, const int * frame_index,
                               navi_frame_result * results);
/* Enqueue-only form of navi_frame_run_batch; navi_frame_collect_batch returns its results. */
int navi_frame_enqueue_batch(navi_frame * f, int nb, const int * slots, navi_kv * const * kvs, const int * n_past,
                             const float * const * d_trailing, const navi_sampling * s, const uint64_t * seeds, const int * frame_index);
int navi_frame_collect_batch(navi_frame * f, int nb, navi_frame_result * results);
const float * navi_frame_step_out_slot(const navi_frame * f, int slot);
int navi_frame_set_step_in_slot(navi_frame * f, int slot, const float * d_step);
/* As navi_frame_inspect, for stream `index` of the last launch. */
int navi_frame_inspect_stream(const navi_frame * f, int index, float * h_hidden, float * h_logits, float * h_clogits);
void navi_frame_destroy(navi_frame * f);

/* ---- graph: replaces navi::qwen3tts::Graph (model/qwen3tts/graph.h:22-79) ---------------- */

typedef struct navi_graph navi_graph;

typedef struct navi_synth_stats {   /* SynthStats, graph.h:43-48 */
    int n_tokens, n_frames, hit_cap, eos;
    double prefill_ms, frames_ms, total_ms;
    double ttfc_ms;                 /* time to the first frame's codes */
    double vocoder_ms;              /* wall time inside vocoder calls */
    double ttfa_ms;                 /* time to the first PCM batch (0 for navi_graph_synth_ids) */
    double audio_s, rtf;            /* n_frames * codec_upsample / sample_rate; total_ms / 1000 / audio_s */
} navi_synth_stats;

/* Graph::load (graph.cpp:22-44) minus the tokenizer and speaker encoder: a talker (prompts up
 * to max_prompt_tokens, KV for max_prompt_tokens + max_frames + 1 positions), a frame kernel
 * and, for vocoder_chunk > 0, a vocoder of vocoder_chunk frames per pass (the reference's
 * vocoder_chunk argument, default 32) on the uploaded weights. */
int navi_graph_create(navi_device * dev, const navi_weights * w, const navi_frame_opts * opts, int max_prompt_tokens, int max_frames,
                      int vocoder_chunk, navi_graph ** out);
/* Codes only: the loop of Graph::synth (graph.cpp:52-111) from token ids (see
 * navi_talker_build_prompt) without the vocoder; writes the 16 codes of each frame to
 * codes[16 * i] (room for codes_cap frames) until EOS or max_frames. */
int navi_graph_synth_ids(navi_graph * g, const int32_t * ids, int n_ids, const char * language, const float * speaker,
                         const navi_sampling * s, uint64_t seed, int max_frames, int32_t * codes, int codes_cap, navi_synth_stats * st);

/* Receives one vocoder batch of 24 kHz f32 PCM (valid during the call only). */
typedef void (*navi_pcm_fn)(const float * pcm, int n_samples, void * user);
/* Graph::synth (graph.cpp:52-111) with audio: as navi_graph_synth_ids, and the frames go
 * through the vocoder in batches of first_batch, then vocoder_batch frames (0 = the
 * vocoder's chunk; SynthRequest::first_batch / vocoder_batch, graph.h:39-40) with each
 * batch's PCM handed to on_pcm. codes may be NULL (codes_cap is then ignored and max_frames
 * alone bounds the loop). NAVI_E_ARG for a graph created without a vocoder. */
int navi_graph_synth(navi_graph * g, const int32_t * ids, int n_ids, const char * language, const float * speaker,
                     const navi_sampling * s, uint64_t seed, int max_frames, int first_batch, int vocoder_batch, int32_t * codes,
                     int codes_cap, navi_pcm_fn on_pcm, void * user, navi_synth_stats * st);
void navi_graph_destroy(navi_graph * g);

/* ---- several utterances at once (no counterpart in the reference, which synthesises one
 *      request at a time, server.cpp:32-84) ---- */
/* As navi_graph_create, for up to max_streams (1..4) utterances per navi_graph_synth_batch
 * call: one talker (KV cache) and one vocoder per stream, one frame kernel. */
int navi_graph_create_streams(navi_device * dev, const navi_weights * w, const navi_frame_opts * opts, int max_prompt_tokens,
                              int max_frames, int vocoder_chunk, int max_streams, navi_graph ** out);
typedef struct navi_synth_request { /* one utterance of a batch (SynthRequest, graph.h:32-41, per stream) */
    const int32_t * ids;
    int n_ids;
    const char * language;
    const float * speaker;          /* host [hidden] */
    uint64_t seed;
    int max_frames;
    int32_t * codes;                /* optional: room for codes_cap frames x 16 */
    int codes_cap;
} navi_synth_request;
/* Receives one vocoder batch of stream `stream` (its index in the request array). */
typedef void (*navi_stream_pcm_fn)(int stream, const float * pcm, int n_samples, void * user);
/* Graph::synth for n requests (1..max_streams) at once: prompts and prefills one after
 * another, then the running streams decode their frames together (navi_frame_run_batch,
 * 4 / 2 / 1 streams per launch), each until its EOS or max_frames, with its frames vocoded
 * in batches of first_batch then vocoder_batch on its own vocoder. Shared sampling settings;
 * stats[i] per stream, times from the start of the call. on_pcm may be NULL (codes only). */
int navi_graph_synth_batch(navi_graph * g, int n, const navi_synth_request * reqs, const navi_sampling * s, int first_batch,
                           int vocoder_batch, navi_stream_pcm_fn on_pcm, void * user, navi_synth_stats * stats);

/* ---- vocoder: replaces navi::qwen3tts::Vocoder (model/qwen3tts/vocoder.h:27-55) ----------- */

typedef struct navi_vocoder navi_vocoder;

/* Vocoder::create (vocoder.hip:413-610): packs the codec decoder's weights into tensor-core
 * tiles and sizes the scratch for chunks of up to max_chunk_frames frames. max_frames is
 * accepted for interface parity (the attention ring needs window + max_chunk_frames rows). */
int navi_vocoder_create(navi_device * dev, const navi_weights * w, int max_chunk_frames, int max_frames, navi_vocoder ** out);
/* Vocoder::reset (vocoder.hip:612-630): zero every conv history and the position (new utterance). */
int navi_vocoder_reset(navi_vocoder * v);
/* Vocoder::decode (vocoder.hip:632-651): codes [n_frames][n_q] (host) -> n_frames *
 * samples_per_frame f32 samples in [-1, 1] written to h_pcm (host, room for cap floats).
 * Decodes in chunks of max_chunk_frames; state carries over to the next call. Code ids outside
 * the codebook return NAVI_E_ARG before anything runs. */
int navi_vocoder_decode(navi_vocoder * v, const int32_t * h_codes, int n_frames, float * h_pcm, size_t cap);
int navi_vocoder_samples_per_frame(const navi_vocoder * v);
int navi_vocoder_max_chunk_frames(const navi_vocoder * v);
/* Vocoder::last_ms: device time of the last decode call (copies included). */
double navi_vocoder_last_ms(const navi_vocoder * v);
/* Vocoder::set_stage_hook (vocoder.h:50-53): fn(user, name, d_buf, rows, cols) after each stage
 * (rvq, pre_conv, layer<l>, pre_transformer, up<j>, dec0, dec<b>, pcm), stream synchronised;
 * d_buf is a device buffer valid during the call. fn NULL removes the hook. */
typedef void (*navi_stage_fn)(void * user, const char * name, const float * d_buf, int rows, int cols);
int navi_vocoder_set_stage_hook(navi_vocoder * v, navi_stage_fn fn, void * user);
void navi_vocoder_destroy(navi_vocoder * v);

/* The implicit-GEMM causal Conv1d of the vocoder on its own (the reference's k_conv,
 * kernels.h:72-242, with its ConvArgs), on device buffers:
 *   y[t][co] = epi(bias[co] + sum_j sum_ci W[co][ci][j] * pro(x~[t - (K-1-j) dil][ci]))
 * with x~ = the T input rows (row stride x_stride) preceded by the H = (K-1) dil rows of hist
 * ([H][Cin], NULL = zeros). trans_stride > 0 instead takes w as a ConvTranspose1d weight
 * [Cin][Cout][K * trans_stride] of that stride, giving output rows t * stride + phase
 * (vocoder.hip:373-385; y must then be dense, y_stride = Cout * stride). Prologue: 0 none,
 * 1 SnakeBeta (snake_a = e^alpha, snake_b = 1/(e^beta + 1e-9)), 2 silu(x[:, :Cin]) *
 * x[:, Cin:2Cin]. Epilogue: 0 none, 1 erf GELU, 2 + resid, 3 * scale + resid (resid rows
 * [T][y_stride]), 4 SiLU. Cin % 8 == 0, x_stride % 4 == 0, 16-byte aligned x / hist. Packs the weight
 * and allocates its workspace on every call: a primitive for tests and tools, not the hot path. */
typedef struct navi_conv_args {
    const uint16_t * w;            /* f16 bits */
    int Cout, Cin, K, dil, trans_stride;
    const float * x; int x_stride, T;
    const float * hist;
    int pro; const float * snake_a, * snake_b;
    int epi; const float * bias, * resid, * scale;
    float * y; int y_stride;
    int rowmajor;                  /* K == 1 only: w is the layer's own row-major [Cout][Cin] matrix, read by
                                      TMA in 128B-swizzled boxes with no packed copy (the path the prefill uses) */
} navi_conv_args;
int navi_conv1d(navi_device * dev, const navi_conv_args * a);

/* Inspection of the last frame (host copies): the talker's post-norm hidden [hidden],
 * its codec logits [talker vocab], and the 15 code-predictor logit rows [15][cp vocab].
 * Any pointer may be NULL. The reference keeps these in its Work buffers (frame.hip:51-70). */
int navi_frame_inspect(const navi_frame * f, float * h_hidden, float * h_logits, float * h_clogits);

/* Phase trace (the reference's NAVI_FRAME_PROFILE, frame.hip:522-529, 612-650, made a
 * runtime switch): when enabled, CTA `cta` (every CTA if cta < 0) records %globaltimer (ns)
 * at the start of each launch and four stamps per phase (inputs ready, weights ready, dot
 * products done, end). navi_frame_profile copies the last launch's trace, one block of
 * 4 * phases + 1 words per traced CTA (as many whole blocks as `cap` holds): block[0] =
 * start, block[1 + 4p + k] = stamp k of phase p; *n = the words written. */
int navi_frame_set_profile(navi_frame * f, int enable, int cta);
int navi_frame_profile(const navi_frame * f, uint64_t * out, int cap, int * n);

/* The device sampler alone, on device logits (one CTA), for parity checks of the
 * draw: codebook 0 applies the codebook-0 modifications with `seen` (device u8[V]
 * or NULL). Writes the chosen id to *out. */
int navi_sample_logits(navi_device * dev, const float * d_logits, int vocab, const navi_sampling * s, uint64_t seed,
                       int frame_index, int codebook, int suppress_from, int eos_id, const uint8_t * d_seen, int32_t * out);

/* No counterpart in the reference.  navi_sample_logits without any device allocation, for
 * hosts that may not allocate after start-up (real-time audio threads, memory-reserved
 * serving processes): the working arrays and the result word live in one static device
 * array of the library (NAVI_SAMPLE_STATIC_MAX_VOCAB logits, about 515 KB).  Same
 * arguments and result as navi_sample_logits; vocab above the limit returns NAVI_E_ARG.
 * The first call on a device takes the array's address (set-up) and should precede any
 * stream capture there.  Calls on one device share the array: the library serialises them
 * with a per-device host lock, and overlapping use of the array by other means races. */
#define NAVI_SAMPLE_STATIC_MAX_VOCAB 32768
int navi_sample_logits_static(navi_device * dev, const float * d_logits, int vocab, const navi_sampling * s, uint64_t seed,
                              int frame_index, int codebook, int suppress_from, int eos_id, const uint8_t * d_seen,
                              int32_t * out);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* NAVI_B200_H */
