// The packed resident weight layout shared by the batch-1 qmv (qmv_packed.cu) and the
// batched decode qmv (qmv_batched.cu), and the GeGLU epilogue both apply.
//
// Rows are grouped in 16-row blocks (zero padded), K in 512-wide units of 8 groups of
// 64 codes (the last unit may hold fewer). For row block rb and unit u the item is one
// contiguous run of nv * 144 bytes, nv = 8 * ceil(gc / 2) valid lanes: chunk c (0..7)
// of every valid lane, then one 16-byte scale/bias record per lane. Lane (g, t) owns
// rows g and g + 8 and groups 2t, 2t + 1 of the unit; chunk c = (row h = c / 4, 16-byte
// piece c % 4 of its 64-byte segment: pieces 0-1 group 2t, pieces 2-3 group 2t + 1).
// The record holds bf16 {sA(g), sB(g), sA(g+8), sB(g+8), bA(g), bB(g), bA(g+8), bB(g+8)}.
// Lane rank = g * tv + t with tv = ceil(gc / 2).
#pragma once

#include "common.cuh"

namespace hyb {

constexpr int kItemMax = 32 * 144;  // bytes of one full item (4608)

struct PackGeo {
    int K, N, G, nunits, nrb;
    int gc_last, tv_last, item_last;  // last unit's group count, valid t count, bytes
    long long rb_bytes;               // bytes of one 16-row block
};

__host__ __device__ inline PackGeo pack_geo(int K, int N) {
    PackGeo p;
    p.K = K;
    p.N = N;
    p.G = K / 64;
    p.nunits = (p.G + 7) / 8;
    p.nrb = (N + 15) / 16;
    p.gc_last = p.G - 8 * (p.nunits - 1);
    p.tv_last = (p.gc_last + 1) / 2;
    p.item_last = 8 * p.tv_last * 144;
    p.rb_bytes = static_cast<long long>(p.nunits - 1) * kItemMax + p.item_last;
    return p;
}

// GELU-tanh built from bf16 elementwise ops, each rounding to bf16 (forward.cc:324-343).
__device__ __forceinline__ float gelu_tanh_bf16ops(float x) {
    const float kC = 0.044677734375f;  // bf16(0.044715)
    const float kK = 0.796875f;        // bf16(sqrt(2/pi))
    float x2 = rbf(x * x);
    float x3 = rbf(x * x2);
    float in = rbf(kC * x3);
    in = rbf(in + x);
    in = rbf(kK * in);
    float th = rbf(tanhf(in));
    float hx = rbf(0.5f * x);
    float op = rbf(1.0f + th);
    return rbf(hx * op);
}

// Named barrier over `count` threads (a team of warps); id 0 is __syncthreads.
__device__ __forceinline__ void team_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

}  // namespace hyb
