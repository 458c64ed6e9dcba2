// CPU SIMT shim for compiling the reference's HIP kernels with g++.
//
// TEST INFRASTRUCTURE ONLY (part of the parity oracle).  It lets the
// reference's routed-MoE source (kernels/routed_storage/*.cpp, unmodified
// apart from the mechanical `<<<...>>>` launch-syntax rewrite done by
// oracle/build_ref.py) run on the host so its outputs pin the C restatement.
//
// Execution model: a launch runs every block; blocks are spread over OpenMP
// threads.  The threads of one block are cooperative fibers (ucontext) on one
// OS thread, so __syncthreads, warp shuffles and the wave-wide WMMA builtin are
// barriers between fibers.  __shared__ arrays become thread_local statics,
// which is per-block storage because a block never leaves its OS thread.
//
// AMD builtins are emulated from their documented semantics:
//   __builtin_amdgcn_sudot8(sa, a, sb, b, c, clamp): c + sum of 8 products of
//       4-bit lanes (bits 4i..4i+3), each operand signed or unsigned;
//   __builtin_amdgcn_wmma_i32_16x16x16_iu4_w32(sa, A, sb, B, C, clamp): wave32
//       16x16x16 integer MMA; lane l holds row l%16 of A and column l%16 of B
//       as 16 nibbles in two dwords (k = 8*dword + nibble); D element (m, n) is
//       in lane n + 16*(m&1), dword m>>1;
//   __builtin_amdgcn_sudot4(sa, a, sb, b, c, clamp): c + sum of 4 products of
//       8-bit lanes (byte i = bits 8i..8i+7), each operand signed or unsigned;
//   __builtin_amdgcn_wmma_i32_16x16x16_iu8_w32(sa, A, sb, B, C, clamp): as the
//       iu4 form with 16 bytes per lane in four dwords (k = 4*dword + byte);
//   __builtin_amdgcn_readfirstlane(v): lane 0's value.
#pragma once
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <ucontext.h>
#include <functional>
#include <vector>
#include "hip_runtime_api.h"
#include "hip_fp16.h"

#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __launch_bounds__(...)
#define __shared__ static thread_local
// clang's ext_vector_type becomes a GCC vector of int32 (every use here is int32_t).
#define ext_vector_type(n) vector_size(4 * (n))

struct dim3 {
    unsigned x, y, z;
    dim3(unsigned a = 1, unsigned b = 1, unsigned c = 1) : x(a), y(b), z(c) {}
};

namespace hipshim {

constexpr int kStack = 64 * 1024;

struct Fiber {
    ucontext_t ctx;
    unsigned tid = 0;
    bool done = false;
    std::vector<char> stack;
};

struct Block {
    std::vector<Fiber> fibers;
    ucontext_t sched;
    int live = 0;
    int arrived = 0;
    unsigned long generation = 0;
    int current = 0;
    const std::function<void()>* body = nullptr;
    // per-warp exchange buffers
    std::vector<uint32_t> xch;
    std::vector<int32_t> wa, wb;  // WMMA operands: 32 lanes x up to 4 dwords each
};

inline thread_local Block* g_block = nullptr;
inline thread_local dim3 g_blockIdx, g_blockDim, g_gridDim;

inline dim3 current_tid() { return dim3(g_block->fibers[g_block->current].tid, 0, 0); }

inline void yield() {
    Block* b = g_block;
    Fiber& f = b->fibers[b->current];
    swapcontext(&f.ctx, &b->sched);
}

inline void release_if_complete(Block* b) {
    if (b->arrived > 0 && b->arrived == b->live) {
        b->arrived = 0;
        b->generation++;
    }
}

// Block-wide barrier among the fibers that have not exited.
inline void barrier() {
    Block* b = g_block;
    unsigned long gen = b->generation;
    b->arrived++;
    release_if_complete(b);
    while (b->generation == gen) yield();
}

inline void trampoline() {
    Block* b = g_block;
    (*b->body)();
    b->fibers[b->current].done = true;
    b->live--;
    release_if_complete(b);
    swapcontext(&b->fibers[b->current].ctx, &b->sched);
}

inline void run_block(const std::function<void()>& body, unsigned nthreads) {
    Block blk;
    blk.body = &body;
    blk.fibers.resize(nthreads);
    blk.live = (int)nthreads;
    blk.xch.assign(nthreads + 32, 0);
    blk.wa.assign((nthreads + 32) * 4, 0);
    blk.wb.assign((nthreads + 32) * 4, 0);
    Block* saved = g_block;
    g_block = &blk;
    for (unsigned t = 0; t < nthreads; ++t) {
        Fiber& f = blk.fibers[t];
        f.tid = t;
        f.stack.resize(kStack);
        getcontext(&f.ctx);
        f.ctx.uc_stack.ss_sp = f.stack.data();
        f.ctx.uc_stack.ss_size = f.stack.size();
        f.ctx.uc_link = nullptr;
        makecontext(&f.ctx, (void (*)())trampoline, 0);
    }
    int remaining = (int)nthreads;
    while (remaining > 0) {
        for (unsigned t = 0; t < nthreads; ++t) {
            if (blk.fibers[t].done) continue;
            blk.current = (int)t;
            swapcontext(&blk.sched, &blk.fibers[t].ctx);
            if (blk.fibers[t].done) remaining--;
        }
    }
    g_block = saved;
}

struct Launch {
    dim3 grid, block;
    Launch(dim3 g, dim3 b, size_t, hipStream_t) : grid(g), block(b) {}
    template <class F, class... A>
    void operator()(F kernel, A... args) {
        const long nblocks = (long)grid.x * grid.y * grid.z;
        const unsigned nthreads = block.x * block.y * block.z;
        const dim3 grid_copy = grid, block_copy = block;
#pragma omp parallel for schedule(dynamic, 1)
        for (long bi = 0; bi < nblocks; ++bi) {
            g_gridDim = grid_copy;
            g_blockDim = block_copy;
            g_blockIdx = dim3((unsigned)bi, 0, 0);
            std::function<void()> body = [&]() { kernel(args...); };
            run_block(body, nthreads);
        }
    }
};

inline unsigned lane_id() { return g_block->fibers[g_block->current].tid & 31u; }
inline unsigned warp_base() { return g_block->fibers[g_block->current].tid & ~31u; }

template <class T>
inline T shfl(T v, int src, int width) {
    static_assert(sizeof(T) == 4, "32-bit shuffles only");
    Block* b = g_block;
    unsigned lane = lane_id(), base = warp_base();
    uint32_t bits;
    memcpy(&bits, &v, 4);
    b->xch[base + lane] = bits;
    barrier();
    unsigned w = (unsigned)width;
    unsigned s = (lane & ~(w - 1)) + ((unsigned)src & (w - 1));
    uint32_t got = b->xch[base + s];
    barrier();
    T out;
    memcpy(&out, &got, 4);
    return out;
}

inline int nib(uint32_t word, int i, bool is_signed) {
    int v = (int)((word >> (4 * i)) & 15u);
    return (is_signed && v >= 8) ? v - 16 : v;
}

inline int byte8(uint32_t word, int i, bool is_signed) {
    int v = (int)((word >> (8 * i)) & 255u);
    return (is_signed && v >= 128) ? v - 256 : v;
}

}  // namespace hipshim

#define threadIdx (::hipshim::current_tid())
#define blockIdx (::hipshim::g_blockIdx)
#define blockDim (::hipshim::g_blockDim)
#define gridDim (::hipshim::g_gridDim)

inline void __syncthreads() { ::hipshim::barrier(); }
template <class T>
inline T __shfl(T v, int src, int width = 32) { return ::hipshim::shfl(v, src, width); }
template <class T>
inline T __shfl_xor(T v, int mask, int width = 32) {
    return ::hipshim::shfl(v, (int)(::hipshim::lane_id() ^ (unsigned)mask), width);
}

inline unsigned atomicOr(unsigned* p, unsigned v) { return __atomic_fetch_or(p, v, __ATOMIC_SEQ_CST); }
inline int atomicAdd(int* p, int v) { return __atomic_fetch_add(p, v, __ATOMIC_SEQ_CST); }
inline unsigned atomicAdd(unsigned* p, unsigned v) { return __atomic_fetch_add(p, v, __ATOMIC_SEQ_CST); }

inline float __uint_as_float(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
inline uint32_t __float_as_uint(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
inline float __fdiv_rn(float a, float b) { return a / b; }
inline int __float2int_rn(float x) { return (int)nearbyintf(x); }

inline int hipshim_sudot8(bool sa, int a, bool sb, int b, int c, bool) {
    int acc = c;
    for (int i = 0; i < 8; ++i) acc += ::hipshim::nib((uint32_t)a, i, sa) * ::hipshim::nib((uint32_t)b, i, sb);
    return acc;
}
#define __builtin_amdgcn_sudot8 hipshim_sudot8

template <class T>
inline T hipshim_readfirstlane(T v) { return ::hipshim::shfl(v, 0, 32); }
#define __builtin_amdgcn_readfirstlane hipshim_readfirstlane

typedef int32_t hipshim_i32x2 __attribute__((vector_size(8)));
typedef int32_t hipshim_i32x8 __attribute__((vector_size(32)));
inline hipshim_i32x8 hipshim_wmma_iu4(bool sa, hipshim_i32x2 A, bool sb, hipshim_i32x2 B, hipshim_i32x8 C, bool) {
    using namespace ::hipshim;
    Block* blk = g_block;
    unsigned lane = lane_id(), base = warp_base();
    blk->wa[2 * (base + lane)] = A[0];
    blk->wa[2 * (base + lane) + 1] = A[1];
    blk->wb[2 * (base + lane)] = B[0];
    blk->wb[2 * (base + lane) + 1] = B[1];
    barrier();
    hipshim_i32x8 D = C;
    unsigned n = lane & 15u, half = lane >> 4;
    for (int v = 0; v < 8; ++v) {
        unsigned m = 2u * (unsigned)v + half;
        int acc = 0;
        for (int k = 0; k < 16; ++k) {
            uint32_t aw = (uint32_t)blk->wa[2 * (base + m) + k / 8];
            uint32_t bw = (uint32_t)blk->wb[2 * (base + n) + k / 8];
            acc += nib(aw, k % 8, sa) * nib(bw, k % 8, sb);
        }
        D[v] += acc;
    }
    barrier();
    return D;
}
#define __builtin_amdgcn_wmma_i32_16x16x16_iu4_w32 hipshim_wmma_iu4

inline int hipshim_sudot4(bool sa, int a, bool sb, int b, int c, bool) {
    int acc = c;
    for (int i = 0; i < 4; ++i) acc += ::hipshim::byte8((uint32_t)a, i, sa) * ::hipshim::byte8((uint32_t)b, i, sb);
    return acc;
}
#define __builtin_amdgcn_sudot4 hipshim_sudot4

typedef int32_t hipshim_i32x4 __attribute__((vector_size(16)));
inline hipshim_i32x8 hipshim_wmma_iu8(bool sa, hipshim_i32x4 A, bool sb, hipshim_i32x4 B, hipshim_i32x8 C, bool) {
    using namespace ::hipshim;
    Block* blk = g_block;
    unsigned lane = lane_id(), base = warp_base();
    for (int d = 0; d < 4; ++d) {
        blk->wa[4 * (base + lane) + d] = A[d];
        blk->wb[4 * (base + lane) + d] = B[d];
    }
    barrier();
    hipshim_i32x8 D = C;
    unsigned n = lane & 15u, half = lane >> 4;
    for (int v = 0; v < 8; ++v) {
        unsigned m = 2u * (unsigned)v + half;
        int acc = 0;
        for (int k = 0; k < 16; ++k) {
            uint32_t aw = (uint32_t)blk->wa[4 * (base + m) + k / 4];
            uint32_t bw = (uint32_t)blk->wb[4 * (base + n) + k / 4];
            acc += byte8(aw, k % 4, sa) * byte8(bw, k % 4, sb);
        }
        D[v] += acc;
    }
    barrier();
    return D;
}
#define __builtin_amdgcn_wmma_i32_16x16x16_iu8_w32 hipshim_wmma_iu8

inline hipError_t hipMemsetAsync(void* p, int v, size_t n, hipStream_t) { memset(p, v, n); return hipSuccess; }
inline hipError_t hipGetLastError() { return hipSuccess; }
