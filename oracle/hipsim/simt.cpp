// Fiber scheduler of the host SIMT emulator (simt.hpp): test infrastructure only.
#include "simt.hpp"

#include <cstdio>
#include <cstdlib>
#include <memory>
#include <vector>

extern "C" void simt_ctx_switch(void ** save_sp, void * load_sp);

// Saves the callee-saved registers of the System V x86-64 ABI on the current stack, stores
// the stack pointer to *save_sp, switches to load_sp and restores the registers saved there.
asm(R"(
    .text
    .globl simt_ctx_switch
    .type simt_ctx_switch, @function
simt_ctx_switch:
    pushq %rbp
    pushq %rbx
    pushq %r12
    pushq %r13
    pushq %r14
    pushq %r15
    movq %rsp, (%rdi)
    movq %rsi, %rsp
    popq %r15
    popq %r14
    popq %r13
    popq %r12
    popq %rbx
    popq %rbp
    ret
    .size simt_ctx_switch, .-simt_ctx_switch
)");

namespace simt {

Thread * g_cur = nullptr;
Dim g_block_idx, g_block_dim, g_grid_dim;

namespace {

enum class State { Runnable, AtBarrier, AtCollective, Done };

struct Fiber {
    Thread t;
    State state = State::Runnable;
    void * sp = nullptr;
    std::unique_ptr<uint8_t[]> stack;
    Coll kind = Coll::None;
    uint64_t bits = 0, result = 0;
    int arg = 0, width = WAVE;
};

constexpr size_t STACK_BYTES = 256 << 10;

struct Block {
    std::vector<Fiber> f;
    void * sched_sp = nullptr;
    int cur = -1;
    const std::function<void()> * body = nullptr;
};

Block * g_blk = nullptr;

[[noreturn]] void die(const char * what) {
    std::fprintf(stderr, "simt: %s (thread %d)\n", what, g_blk ? g_blk->cur : -1);
    std::abort();
}

void yield_to_scheduler() {
    Fiber & me = g_blk->f[static_cast<size_t>(g_blk->cur)];
    simt_ctx_switch(&me.sp, g_blk->sched_sp);
}

void fiber_entry() {
    (*g_blk->body)();
    g_blk->f[static_cast<size_t>(g_blk->cur)].state = State::Done;
    yield_to_scheduler();
    die("a finished fiber was resumed");
}

// Releases the block barrier when every live fiber waits at it.
bool try_release_barrier() {
    bool any = false;
    for (Fiber & x : g_blk->f) {
        if (x.state == State::Done) continue;
        if (x.state != State::AtBarrier) return false;
        any = true;
    }
    if (!any) return false;
    for (Fiber & x : g_blk->f)
        if (x.state == State::AtBarrier) x.state = State::Runnable;
    return true;
}

// Completes the collective of wave w when every live lane waits at one.
bool try_release_wave(int w) {
    const int n = static_cast<int>(g_blk->f.size());
    const int l0 = w * WAVE, l1 = l0 + WAVE < n ? l0 + WAVE : n;
    Coll kind = Coll::None;
    for (int i = l0; i < l1; ++i) {
        const Fiber & x = g_blk->f[static_cast<size_t>(i)];
        if (x.state == State::Done) continue;
        if (x.state != State::AtCollective) return false;
        if (kind == Coll::None) kind = x.kind;
        else if (kind != x.kind) die("lanes of one wavefront reached different collectives");
    }
    if (kind == Coll::None) return false;
    uint64_t ballot = 0;
    for (int i = l0; i < l1; ++i) {
        const Fiber & x = g_blk->f[static_cast<size_t>(i)];
        if (x.state == State::AtCollective && x.bits) ballot |= 1ull << (i - l0);
    }
    for (int i = l0; i < l1; ++i) {
        Fiber & x = g_blk->f[static_cast<size_t>(i)];
        if (x.state != State::AtCollective) continue;
        const int lane = i - l0, seg = lane & ~(x.width - 1);
        int src = lane;
        switch (kind) {
            case Coll::ShflXor: src = lane ^ x.arg; break;
            case Coll::ShflUp: src = lane - x.arg < seg ? lane : lane - x.arg; break;
            case Coll::ShflIdx: src = seg + (x.arg & (x.width - 1)); break;
            default: break;
        }
        if (kind == Coll::Ballot) {
            x.result = ballot;
        } else {
            if (src < 0 || l0 + src >= l1) die("shuffle source lane outside the wavefront");
            const Fiber & s = g_blk->f[static_cast<size_t>(l0 + src)];
            if (s.state != State::AtCollective) die("shuffle reads a lane that has exited");
            x.result = s.bits;
        }
    }
    for (int i = l0; i < l1; ++i) {
        Fiber & x = g_blk->f[static_cast<size_t>(i)];
        if (x.state == State::AtCollective) x.state = State::Runnable;
    }
    return true;
}

} // namespace

void block_barrier() {
    Fiber & me = g_blk->f[static_cast<size_t>(g_blk->cur)];
    me.state = State::AtBarrier;
    yield_to_scheduler();
}

uint64_t wave_collective(Coll kind, uint64_t bits, int arg, int width) {
    Fiber & me = g_blk->f[static_cast<size_t>(g_blk->cur)];
    if (width <= 0 || width > WAVE || (width & (width - 1))) die("collective width must be a power of two <= 32");
    me.kind = kind;
    me.bits = bits;
    me.arg = arg;
    me.width = width;
    me.state = State::AtCollective;
    yield_to_scheduler();
    return g_blk->f[static_cast<size_t>(g_blk->cur)].result;
}

void run_block(unsigned threads, Dim block_idx, Dim grid, const std::function<void()> & body) {
    Block blk;
    blk.body = &body;
    blk.f.resize(threads);
    g_block_idx = block_idx;
    g_grid_dim = grid;
    g_block_dim = Dim{threads, 1, 1};
    for (unsigned i = 0; i < threads; ++i) {
        Fiber & x = blk.f[i];
        x.t.tid = Dim{i, 0, 0};
        x.stack.reset(new uint8_t[STACK_BYTES]);
        // initial frame: six zeroed callee-saved registers, then fiber_entry as the return
        // address, placed so that fiber_entry starts with the ABI's call-site alignment
        uintptr_t top = reinterpret_cast<uintptr_t>(x.stack.get() + STACK_BYTES) & ~uintptr_t(15);
        uintptr_t ret_slot = top - 16;
        reinterpret_cast<void **>(ret_slot)[0] = reinterpret_cast<void *>(&fiber_entry);
        reinterpret_cast<void **>(ret_slot)[1] = nullptr;
        for (int r = 1; r <= 6; ++r) reinterpret_cast<void **>(ret_slot)[-r] = nullptr;
        x.sp = reinterpret_cast<void *>(ret_slot - 6 * sizeof(void *));
    }
    Block * prev = g_blk;
    g_blk = &blk;
    const int n = static_cast<int>(threads);
    const int nw = (n + WAVE - 1) / WAVE;
    for (;;) {
        bool ran = false;
        for (int i = 0; i < n; ++i) {
            Fiber & x = blk.f[static_cast<size_t>(i)];
            if (x.state != State::Runnable) continue;
            blk.cur = i;
            g_cur = &x.t;
            simt_ctx_switch(&blk.sched_sp, x.sp);
            ran = true;
            if (x.state == State::AtCollective) try_release_wave(i / WAVE);
        }
        bool released = false;
        for (int w = 0; w < nw; ++w) released |= try_release_wave(w);
        released |= try_release_barrier();
        bool all_done = true;
        for (const Fiber & x : blk.f) all_done &= x.state == State::Done;
        if (all_done) break;
        if (!ran && !released) die("deadlock: no fiber can run");
    }
    g_blk = prev;
    g_cur = nullptr;
}

} // namespace simt
