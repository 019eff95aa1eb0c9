// Host runtime: errors, the .navi reader, model parameters and their tensor table,
// the device weight arena, and the device handle.
//
// Interfaces mirror the reference engine's runtime (runtime/common/error.h,
// runtime/weights/navi_file.h, runtime/weights/device_weights.h,
// model/qwen3tts/params.h, runtime/device/device.h) with CUDA in place of HIP.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <string_view>
#include <vector>

namespace navi {

// Setup-time failures throw; the request path returns a status (as in the reference).
struct Error : std::runtime_error {
    int status;
    Error(const std::string & m, int s) : std::runtime_error(m), status(s) {}
};
[[noreturn]] void fail(const std::string & msg, int status = 1);
void cuda_check(cudaError_t e, const char * what, const char * file, int line);
#define NAVI_CUDA(x) ::navi::cuda_check((x), #x, __FILE__, __LINE__)

// ---- .navi v1 ---------------------------------------------------------------------------------

enum class DType : uint8_t { F32 = 0, F16 = 1, BF16 = 2, I32 = 3, U8 = 4 };
size_t dtype_size(DType d);

struct TensorInfo {
    std::string name;
    DType dtype = DType::F32;
    std::vector<uint64_t> dims;
    uint64_t offset = 0, nbytes = 0;
    uint64_t numel() const;
};

struct KV {
    enum class Type : uint8_t { I64 = 0, F64 = 1, STR = 2, I64_ARRAY = 3 };
    Type type = Type::I64;
    int64_t i64 = 0;
    double f64 = 0;
    std::string str;
    std::vector<int64_t> arr;
};

// Releases a read-only file mapping of `bytes` bytes.
struct FileUnmap {
    uint64_t bytes = 0;
    void operator()(const uint8_t * p) const;
};

// A mapped .navi file: the hyperparameters and the tensor table are decoded at open; tensor
// payloads are read in place from the read-only mapping until close() or destruction.
class NaviFile {
public:
    static NaviFile open(const std::string & path);
    NaviFile(NaviFile &&) noexcept = default;
    NaviFile & operator=(NaviFile &&) noexcept = default;
    NaviFile(const NaviFile &) = delete;

    const std::string & path() const { return path_; }
    const std::vector<TensorInfo> & tensors() const { return tensors_; }
    const std::map<std::string, KV> & kv() const { return kv_; }
    bool has_kv(std::string_view k) const;
    int64_t kv_i64(std::string_view k) const;
    int64_t kv_i64_or(std::string_view k, int64_t d) const;
    double kv_f64(std::string_view k) const;
    double kv_f64_or(std::string_view k, double d) const;
    std::string kv_str(std::string_view k) const;
    std::vector<int64_t> kv_i64_array(std::string_view k) const;
    const TensorInfo * find(std::string_view name) const;
    const void * data(const TensorInfo & t) const;
    void close();

private:
    NaviFile() = default;
    std::string path_;
    std::unique_ptr<const uint8_t, FileUnmap> map_;
    uint64_t size_ = 0, data_offset_ = 0;
    std::map<std::string, KV> kv_;
    std::vector<TensorInfo> tensors_;
    std::map<std::string, size_t> index_;
};

// ---- model parameters -------------------------------------------------------------------------

struct TransformerParams {
    int hidden = 0, n_layer = 0, n_head = 0, n_kv_head = 0, head_dim = 0, ff = 0, vocab = 0, max_pos = 0;
    float rms_eps = 0;
    double rope_theta = 0;
};

struct Params {
    std::string name;
    int text_vocab = 0, text_hidden = 0, n_code_groups = 0;
    int im_start_id = 0, im_end_id = 0, assistant_id = 0, tts_bos_id = 0, tts_eos_id = 0, tts_pad_id = 0;
    TransformerParams talker, cp, vocoder;
    int codec_bos_id = 0, codec_eos_id = 0, codec_pad_id = 0;
    int codec_think_id = 0, codec_nothink_id = 0, codec_think_bos_id = 0, codec_think_eos_id = 0;
    std::map<std::string, int> language_ids;
    int codec_sample_rate = 0, codec_upsample = 0;
    int vq_latent = 0, vq_codebook_dim = 0, vq_codebook_size = 0, vq_n_q = 0, vq_n_semantic = 0;
    int decoder_dim = 0, sliding_window = 0;
    std::vector<int> upsample_rates, upsampling_ratios;
    float temperature = 1, top_p = 1, repetition_penalty = 1, cp_temperature = 1, cp_top_p = 1;
    int top_k = 0, cp_top_k = 0;
};

// Reads the KV section (reference: model/qwen3tts/params.cpp:59-130).
Params read_params(const NaviFile & f);

struct ExpectedTensor {
    std::string name;
    std::vector<uint64_t> dims;
};
// Every tensor the engine loads, with its shape (reference: params.cpp:132-284).
std::vector<ExpectedTensor> expected_tensors(const Params & p);

struct Validation {
    std::vector<std::string> missing, shape_mismatch, unused;
    bool ok() const { return missing.empty() && shape_mismatch.empty(); }
};
Validation validate(const NaviFile & f, const Params & p);

// ---- device ---------------------------------------------------------------------------------------

struct DeviceInfo {
    int ordinal = -1;
    std::string name;
    int cc_major = 0, cc_minor = 0, multiprocessors = 0;
    bool cooperative_launch = false;
    size_t smem_optin = 0, l2_bytes = 0, vram_total = 0, vram_free = 0;
};

class Device {
public:
    explicit Device(int ordinal);
    ~Device();
    Device(const Device &) = delete;
    const DeviceInfo & info() const { return info_; }
    cudaStream_t stream() const { return stream_; }
    void make_current() const;

private:
    DeviceInfo info_;
    cudaStream_t stream_ = nullptr;
};

// ---- weights arena (reference: runtime/weights/device_weights.cpp:18-72) ----------------------------

struct DeviceTensor {
    TensorInfo info;
    void * ptr = nullptr;
    template <class T> const T * as() const { return static_cast<const T *>(ptr); }
};

class DeviceWeights {
public:
    using Groups = std::vector<std::vector<std::string>>;
    // Every non-U8 tensor in file order, except that each group is placed
    // consecutively where its first member falls; 256-byte alignment.
    static DeviceWeights * upload(const Device & dev, const NaviFile & f, const Groups & groups);
    ~DeviceWeights();
    const DeviceTensor * find(std::string_view name) const;
    const DeviceTensor & get(std::string_view name) const;
    uint64_t bytes() const { return bytes_; }
    const Params & params() const { return params_; }
    Params params_;

private:
    DeviceWeights() = default;
    void * arena_ = nullptr;
    uint64_t bytes_ = 0;
    int ordinal_ = 0;
    std::map<std::string, DeviceTensor> tensors_;
};

// The adjacency groups the kernels rely on: q/k/v and gate/up of every talker and
// code-predictor layer (reference: Talker::fused_groups, talker.hip:190-198).
DeviceWeights::Groups fused_groups(const Params & p);

} // namespace navi
