// A host SIMT emulator for running GPU device code on the CPU: test infrastructure only.
//
// One thread block runs as blockDim.x cooperative fibers on the calling OS thread, switched
// by a small x86-64 context switch. A fiber runs until it reaches a block barrier or a
// wavefront collective (shuffle, ballot), then the next runnable fiber runs; a barrier
// releases when every live fiber of the block waits at one, a collective when every live
// lane of its 32-lane wavefront waits at one, and the collective's results are then computed
// from all lanes' operands at once. Shared memory is ordinary memory, so device code whose
// correctness rests on barriers and collectives runs here with the same results; atomics
// are plain read-modify-writes (fibers never interleave inside one).
//
// Used by oracle/ref_frame_check.cpp to run the reference engine's device functions on the
// host (the reference is HIP for RDNA3 and has no other way to run here).
#pragma once

#include <cstdint>
#include <functional>

namespace simt {

struct Dim {
    unsigned x = 1, y = 1, z = 1;
};

constexpr int WAVE = 32;

enum class Coll : int { None, ShflXor, ShflUp, ShflIdx, Ballot };

// Per-thread state visible to the device code (through the macros of hip_runtime.h).
struct Thread {
    Dim tid;
};

extern Thread * g_cur;
extern Dim g_block_idx, g_block_dim, g_grid_dim;

// __syncthreads()
void block_barrier();
// A wavefront collective: every live lane of the caller's wave passes its operand; returns
// this lane's result (bits of the value read from the source lane, or the ballot mask).
uint64_t wave_collective(Coll kind, uint64_t bits, int arg, int width);

// Runs body() as `threads` fibers of block `block_idx` of a grid of `grid` blocks.
void run_block(unsigned threads, Dim block_idx, Dim grid, const std::function<void()> & body);

} // namespace simt
