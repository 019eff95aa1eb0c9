// Host stand-in for the HIP runtime and device built-ins, so that the reference engine's
// HIP sources compile as plain C++ on the CPU: test infrastructure only (the oracle's
// reference checkers under oracle/_ref).
//
// Device code: qualifiers expand to nothing, threadIdx / blockIdx / blockDim / gridDim read
// the SIMT emulator (simt.hpp), __syncthreads / __shfl_* / __ballot are its barrier and
// wavefront collectives (32 lanes, the RDNA3 wave32 mode the reference is built for),
// atomics are plain read-modify-writes, and the math functions are the host C library's.
// Runtime API: memory calls work on host memory (hipMalloc is malloc, copies are memcpy);
// streams and events do nothing; a cooperative launch runs the kernel through the runner
// the checker registers (simsim::set_launch_runner).
#pragma once

#include "../simt.hpp"

#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <functional>

#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __launch_bounds__(...)
#define __shared__ static
#define __align__(n) __attribute__((aligned(n)))

#define threadIdx (::simt::g_cur->tid)
#define blockIdx (::simt::g_block_idx)
#define blockDim (::simt::g_block_dim)
#define gridDim (::simt::g_grid_dim)
#define warpSize 32

struct dim3 {
    unsigned x, y, z;
    dim3(unsigned a = 1, unsigned b = 1, unsigned c = 1) : x(a), y(b), z(c) {}
};
struct uint4 { unsigned x, y, z, w; };
struct uint2 { unsigned x, y; };
struct float2 { float x, y; };
struct float4 { float x, y, z, w; };
inline uint4 make_uint4(unsigned a, unsigned b, unsigned c, unsigned d) { return uint4{a, b, c, d}; }
inline uint2 make_uint2(unsigned a, unsigned b) { return uint2{a, b}; }
inline float2 make_float2(float a, float b) { return float2{a, b}; }
inline float4 make_float4(float a, float b, float c, float d) { return float4{a, b, c, d}; }
using std::max;
using std::min;

namespace simsim {
template <class T> inline uint64_t to_bits(T v) {
    uint64_t b = 0;
    std::memcpy(&b, &v, sizeof(T));
    return b;
}
template <class T> inline T from_bits(uint64_t b) {
    T v;
    std::memcpy(&v, &b, sizeof(T));
    return v;
}
// kernel launches: fn(grid, block, args)
using LaunchRunner = std::function<int(const void * fn, dim3 grid, dim3 block, void ** args)>;
inline LaunchRunner & launch_runner() {
    static LaunchRunner r;
    return r;
}
inline void set_launch_runner(LaunchRunner r) { launch_runner() = std::move(r); }

// kernel<<<grid, block, smem, stream>>>(args), rewritten by oracle/hip_to_host.py: the blocks of
// the grid run one after another (kernels without inter-block waits only)
struct Launch {
    dim3 grid, block;
    template <class F, class... A> void run(F fn, A &&... args) const {
        for (unsigned z = 0; z < grid.z; ++z)
            for (unsigned y = 0; y < grid.y; ++y)
                for (unsigned x = 0; x < grid.x; ++x)
                    ::simt::run_block(block.x * block.y * block.z, ::simt::Dim{x, y, z}, ::simt::Dim{grid.x, grid.y, grid.z},
                                      [&]() { fn(args...); });
    }
};
inline Launch launch(dim3 grid, dim3 block, size_t = 0, void * = nullptr) { return Launch{grid, block}; }
} // namespace simsim

inline void __syncthreads() { ::simt::block_barrier(); }
inline float __expf(float x) { return std::exp(x); }
inline float __sinf(float x) { return std::sin(x); }
inline void __threadfence() {}
template <class T> inline T __shfl_xor(T v, int mask, int width = 32) {
    return simsim::from_bits<T>(::simt::wave_collective(::simt::Coll::ShflXor, simsim::to_bits(v), mask, width));
}
template <class T> inline T __shfl_up(T v, unsigned delta, int width = 32) {
    return simsim::from_bits<T>(::simt::wave_collective(::simt::Coll::ShflUp, simsim::to_bits(v), static_cast<int>(delta), width));
}
template <class T> inline T __shfl(T v, int src, int width = 32) {
    return simsim::from_bits<T>(::simt::wave_collective(::simt::Coll::ShflIdx, simsim::to_bits(v), src, width));
}
inline unsigned long long __ballot(int pred) { return ::simt::wave_collective(::simt::Coll::Ballot, pred ? 1u : 0u, 0, 32); }
inline int __popcll(unsigned long long v) { return __builtin_popcountll(v); }
inline int __popc(unsigned v) { return __builtin_popcount(v); }
inline unsigned atomicAdd(unsigned * p, unsigned v) {
    const unsigned old = *p;
    *p = old + v;
    return old;
}
inline int atomicAdd(int * p, int v) {
    const int old = *p;
    *p = old + v;
    return old;
}
inline float atomicAdd(float * p, float v) {
    const float old = *p;
    *p = old + v;
    return old;
}
inline unsigned __float_as_uint(float f) { return simsim::from_bits<unsigned>(simsim::to_bits(f)); }
inline float __uint_as_float(unsigned u) { return simsim::from_bits<float>(simsim::to_bits(u)); }
inline float rsqrtf(float x) { return 1.0f / std::sqrt(x); }

// ---- runtime API on host memory ----
enum hipError_t { hipSuccess = 0, hipErrorNoDevice = 100, hipErrorInvalidValue = 1 };
enum hipMemcpyKind { hipMemcpyHostToHost = 0, hipMemcpyHostToDevice = 1, hipMemcpyDeviceToHost = 2, hipMemcpyDeviceToDevice = 3, hipMemcpyDefault = 4 };
enum hipDeviceAttribute_t { hipDeviceAttributeWallClockRate = 0 };
typedef struct ihipStream_t * hipStream_t;
typedef struct ihipEvent_t * hipEvent_t;
constexpr unsigned hipStreamNonBlocking = 1;
constexpr unsigned hipDeviceScheduleSpin = 1;

inline const char * hipGetErrorString(hipError_t) { return "host stand-in for the HIP runtime"; }
inline const char * hipGetErrorName(hipError_t) { return "hipErrorHostStandIn"; }
inline hipError_t hipMemGetInfo(size_t * free_b, size_t * total_b) {
    *free_b = *total_b = size_t(1) << 40;
    return hipSuccess;
}
inline hipError_t hipMalloc(void ** p, size_t n) {
    *p = std::calloc(n ? n : 1, 1);
    return *p ? hipSuccess : hipErrorInvalidValue;
}
inline hipError_t hipFree(void * p) {
    std::free(p);
    return hipSuccess;
}
inline hipError_t hipMemcpy(void * d, const void * s, size_t n, hipMemcpyKind) {
    if (n) std::memmove(d, s, n);
    return hipSuccess;
}
inline hipError_t hipMemcpyAsync(void * d, const void * s, size_t n, hipMemcpyKind k, hipStream_t = nullptr) { return hipMemcpy(d, s, n, k); }
inline hipError_t hipMemset(void * d, int v, size_t n) {
    std::memset(d, v, n);
    return hipSuccess;
}
inline hipError_t hipMemsetAsync(void * d, int v, size_t n, hipStream_t = nullptr) { return hipMemset(d, v, n); }
inline hipError_t hipEventCreate(hipEvent_t * e) {
    *e = nullptr;
    return hipSuccess;
}
inline hipError_t hipEventDestroy(hipEvent_t) { return hipSuccess; }
inline hipError_t hipEventRecord(hipEvent_t, hipStream_t = nullptr) { return hipSuccess; }
inline hipError_t hipEventElapsedTime(float * ms, hipEvent_t, hipEvent_t) {
    *ms = 0.f;
    return hipSuccess;
}
inline hipError_t hipStreamSynchronize(hipStream_t) { return hipSuccess; }
inline hipError_t hipEventSynchronize(hipEvent_t) { return hipSuccess; }
inline hipError_t hipGetLastError() { return hipSuccess; }
inline hipError_t hipDeviceSynchronize() { return hipSuccess; }
inline hipError_t hipDeviceGetAttribute(int * v, hipDeviceAttribute_t, int) {
    *v = 1;
    return hipSuccess;
}
template <class F> inline hipError_t hipOccupancyMaxActiveBlocksPerMultiprocessor(int * n, F, int, size_t) {
    *n = 1;
    return hipSuccess;
}
template <class F> inline hipError_t hipLaunchCooperativeKernel(F fn, dim3 grid, dim3 block, void ** args, size_t, hipStream_t) {
    auto & r = simsim::launch_runner();
    if (!r) return hipErrorInvalidValue;
    return r(reinterpret_cast<const void *>(fn), grid, block, args) == 0 ? hipSuccess : hipErrorInvalidValue;
}
