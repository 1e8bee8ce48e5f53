// Memory-bound helper kernels of the decoder: embedding gather, RMSNorm and its
// residual variants, GeGLU, the QK-norm/RoPE/cache-write prologue of attention,
// ring gathers and the softcap + top-k epilogue of the lm_head.
//
// Rounding follows the reference's MLX op graph: every op whose MLX result is
// bf16 is rounded to bf16 here too (forward.cc:25-27, 126-160, 324-343, 394-420,
// 510-542).
#include "kernels.h"

#include <algorithm>
#include <cfloat>

namespace hyb {
namespace {

__device__ __forceinline__ float block_reduce_sum(float v, float* sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    float r = (lane < nw) ? sh[lane] : 0.f;
    return warp_sum(r);
}

// ------------------------------------------------------------------ embed
// (weights_loader.cc:181-198 gather + dequantize, forward.cc:126-131 scale)
__global__ void embed_kernel(const uint32_t* __restrict__ ids, const uint32_t* __restrict__ w,
                             const bf16* __restrict__ s, const bf16* __restrict__ b, int H,
                             bf16 scale, bf16* __restrict__ out) {
    const int l = blockIdx.y;
    const uint32_t id = ids[l];
    const int G = H / 64;
    const float sc = bf2f(scale);
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < H / 8; j += gridDim.x * blockDim.x) {
        const uint32_t word = w[static_cast<size_t>(id) * (H / 8) + j];
        const int g = (8 * j) / 64;
        const float sv = bf2f(s[static_cast<size_t>(id) * G + g]);
        const float bv = bf2f(b[static_cast<size_t>(id) * G + g]);
        bf16 o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float deq = rbf(fmaf(sv, static_cast<float>((word >> (4 * i)) & 0xF), bv));
            o[i] = f2bf(deq * sc);
        }
        *reinterpret_cast<uint4*>(out + static_cast<size_t>(l) * H + 8 * j) = *reinterpret_cast<uint4*>(o);
    }
}

// ------------------------------------------------------------------ rms norms
__global__ void rms_norm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                bf16* __restrict__ out, int D, float eps) {
    __shared__ float sh[32];
    const bf16* xr = x + static_cast<size_t>(blockIdx.x) * D;
    bf16* orow = out + static_cast<size_t>(blockIdx.x) * D;
    float ss = 0.f;
    for (int k = threadIdx.x; k < D; k += blockDim.x) {
        float v = bf2f(xr[k]);
        ss += v * v;
    }
    const float inv = 1.0f / sqrtf(block_reduce_sum(ss, sh) / static_cast<float>(D) + eps);
    for (int k = threadIdx.x; k < D; k += blockDim.x) {
        float t = rbf(bf2f(xr[k]) * inv);
        orow[k] = w ? f2bf(t * bf2f(w[k])) : f2bf(t);
    }
}

// h = bf16(resid + norm(x, post_w)); h *= scalar; out_h = h; out_n = norm(h, next_w)
__global__ void resid_norm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ post_w,
                                  const bf16* resid, const bf16* __restrict__ scalar, bf16* out_h,
                                  const bf16* __restrict__ next_w, bf16* __restrict__ out_n, int D,
                                  float eps) {
    extern __shared__ float hbuf[];  // [D]
    __shared__ float sh[32];
    const size_t off = static_cast<size_t>(blockIdx.x) * D;
    float ss = 0.f;
    for (int k = threadIdx.x; k < D; k += blockDim.x) {
        float v = bf2f(x[off + k]);
        ss += v * v;
    }
    const float inv = 1.0f / sqrtf(block_reduce_sum(ss, sh) / static_cast<float>(D) + eps);
    const float sc = scalar ? bf2f(scalar[0]) : 1.f;
    float ss2 = 0.f;
    for (int k = threadIdx.x; k < D; k += blockDim.x) {
        float nv = rbf(rbf(bf2f(x[off + k]) * inv) * bf2f(post_w[k]));
        float hv = rbf(bf2f(resid[off + k]) + nv);
        if (scalar) hv = rbf(hv * sc);
        hbuf[k] = hv;
        ss2 += hv * hv;
    }
    const float inv2 = 1.0f / sqrtf(block_reduce_sum(ss2, sh) / static_cast<float>(D) + eps);
    for (int k = threadIdx.x; k < D; k += blockDim.x) {
        const float hv = hbuf[k];
        out_h[off + k] = f2bf(hv);
        if (next_w) out_n[off + k] = f2bf(rbf(hv * inv2) * bf2f(next_w[k]));
    }
}

// The same with every operand in registers: each thread issues its 16-byte loads of x,
// resid, post_w and next_w at once (C chunks of 8 elements, D = 8 * chunks <= 2048 C),
// so a row costs one memory round trip plus two block reductions. Same rounding points.
template <int C>
__global__ void __launch_bounds__(256) resid_norm_vec_kernel(const bf16* __restrict__ x, const bf16* __restrict__ post_w,
                                                             const bf16* resid, const bf16* __restrict__ scalar,
                                                             bf16* out_h, const bf16* __restrict__ next_w,
                                                             bf16* __restrict__ out_n, int D, float eps) {
    __shared__ float sh[32];
    const size_t off = static_cast<size_t>(blockIdx.x) * D;
    const int nch = D / 8;
    const uint4 z = make_uint4(0, 0, 0, 0);
    uint4 xv[C], rv[C], pv[C], nv[C];
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const int j = threadIdx.x + 256 * c;
        const bool ok = j < nch;
        xv[c] = ok ? reinterpret_cast<const uint4*>(x + off)[j] : z;
        rv[c] = ok ? reinterpret_cast<const uint4*>(resid + off)[j] : z;
        pv[c] = ok ? reinterpret_cast<const uint4*>(post_w)[j] : z;
        nv[c] = (ok && next_w) ? reinterpret_cast<const uint4*>(next_w)[j] : z;
    }
    auto el = [](const uint4& v, int e) {  // element e (0..7) of a 16-byte chunk
        const uint32_t w = e < 2 ? v.x : e < 4 ? v.y : e < 6 ? v.z : v.w;
        return __uint_as_float((e & 1) ? (w & 0xFFFF0000u) : (w << 16));
    };
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c)
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += el(xv[c], e) * el(xv[c], e);
    const float inv = 1.0f / sqrtf(block_reduce_sum(ss, sh) / static_cast<float>(D) + eps);
    const float sc = scalar ? bf2f(scalar[0]) : 1.f;
    float hv[C][8];
    float ss2 = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float n = rbf(rbf(el(xv[c], e) * inv) * el(pv[c], e));
            float h = rbf(el(rv[c], e) + n);
            if (scalar) h = rbf(h * sc);
            hv[c][e] = h;
            ss2 += h * h;
        }
    const float inv2 = 1.0f / sqrtf(block_reduce_sum(ss2, sh) / static_cast<float>(D) + eps);
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const int j = threadIdx.x + 256 * c;
        if (j >= nch) continue;
        uint4 ho, no;
        uint32_t* hw = &ho.x;
        uint32_t* nw = &no.x;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            hw[q] = pack_bf2(f2bf(hv[c][2 * q]), f2bf(hv[c][2 * q + 1]));
            nw[q] = pack_bf2(f2bf(rbf(hv[c][2 * q] * inv2) * el(nv[c], 2 * q)),
                             f2bf(rbf(hv[c][2 * q + 1] * inv2) * el(nv[c], 2 * q + 1)));
        }
        reinterpret_cast<uint4*>(out_h + off)[j] = ho;
        if (next_w) reinterpret_cast<uint4*>(out_n + off)[j] = no;
    }
}

// ------------------------------------------------------------------ GeGLU
__device__ __forceinline__ float gelu_tanh_ops(float x) {
    const float kC = 0.044677734375f;  // bf16(0.044715)
    const float kK = 0.796875f;        // bf16(0.7978845608)
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

__global__ void geglu_kernel(const bf16* __restrict__ gate, const bf16* __restrict__ up,
                             bf16* __restrict__ act, int N, int ld_in) {
    const int l = blockIdx.y;
    for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < N; n += gridDim.x * blockDim.x) {
        const float g = bf2f(gate[static_cast<size_t>(l) * ld_in + n]);
        const float u = bf2f(up[static_cast<size_t>(l) * ld_in + n]);
        act[static_cast<size_t>(l) * N + n] = f2bf(gelu_tanh_ops(g) * u);
    }
}

// ------------------------------------------------------------------ QK-norm + RoPE + cache write
// One warp per (token, head) row; heads [0, nh) are q, [nh, nh+nkv) k, [nh+nkv, nh+2nkv) v.
__global__ void qkv_post_kernel(const QkvPostParams p) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int rows_per_tok = p.n_heads + 2 * p.n_kv;
    if (warp >= p.L * rows_per_tok) return;
    const int l = warp / rows_per_tok;
    const int r = warp % rows_per_tok;
    const int hd = p.hd, half = hd / 2;
    const int kind = r < p.n_heads ? 0 : (r < p.n_heads + p.n_kv ? 1 : 2);
    const int head = kind == 0 ? r : (kind == 1 ? r - p.n_heads : r - p.n_heads - p.n_kv);
    int col;
    if (kind == 0) col = head * hd;
    else if (kind == 1 || p.v_from_k) col = p.n_heads * hd + head * hd;
    else col = p.n_heads * hd + p.n_kv * hd + head * hd;
    const bf16* src = p.qkv + static_cast<size_t>(l) * p.ld + col;
    constexpr int kMaxPer = 16;  // hd <= 512
    float v[kMaxPer];
    const int per = hd / 32;
    float ss = 0.f;
    // element e = lane + 32 * i  (i < per); pairs (e, e + half) live in the same lane when
    // half is a multiple of 32, i.e. i and i + per/2.
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
        if (i < per) {
            v[i] = bf2f(src[lane + 32 * i]);
            ss += v[i] * v[i];
        }
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(hd) + p.eps);
    const bf16* nw = kind == 0 ? p.q_norm : (kind == 1 ? p.k_norm : nullptr);
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
        if (i < per) {
            float t = rbf(v[i] * inv);
            v[i] = nw ? rbf(t * bf2f(nw[lane + 32 * i])) : t;
        }
    }
    const int pos = p.pos0 + l;
    if (kind != 2) {
        const int hp = per / 2;
#pragma unroll
        for (int i = 0; i < kMaxPer / 2; ++i) {
            if (i < hp) {
                const int e = lane + 32 * i;  // < half
                const float f = p.inv_freq[e];
                if (f != 0.f) {
                    const float ang = __fmul_rn(static_cast<float>(pos), f);
                    float sn, cs;
                    sincosf(ang, &sn, &cs);
                    const float x1 = v[i], x2 = v[i + hp];
                    v[i] = rbf(x1 * cs - x2 * sn);
                    v[i + hp] = rbf(x1 * sn + x2 * cs);
                }
            }
        }
    }
    bf16* dst = nullptr;
    bf16* cdst = nullptr;
    if (kind == 0) {
        dst = p.q_out + (static_cast<size_t>(l) * p.n_heads + head) * hd;
    } else {
        bf16* contig = kind == 1 ? p.k_out : p.v_out;
        if (contig) dst = contig + (static_cast<size_t>(l) * p.n_kv + head) * hd;
        bf16* cache = kind == 1 ? p.k_cache : p.v_cache;
        if (cache && l >= p.cache_first) {
            const int slot = pos % p.cache_cap;
            cdst = cache + (static_cast<size_t>(slot) * p.n_kv + head) * hd;
        }
    }
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
        if (i < per) {
            const bf16 o = f2bf(v[i]);
            if (dst) dst[lane + 32 * i] = o;
            if (cdst) cdst[lane + 32 * i] = o;
        }
    }
}

__global__ void gather_ring_kernel(const bf16* __restrict__ cache, int cap, int pos0, int n, int row_elems,
                                   bf16* __restrict__ dst) {
    const int j = blockIdx.y;
    const int slot = (pos0 + j) % cap;
    const uint4* s = reinterpret_cast<const uint4*>(cache + static_cast<size_t>(slot) * row_elems);
    uint4* d = reinterpret_cast<uint4*>(dst + static_cast<size_t>(j) * row_elems);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < row_elems / 8; i += gridDim.x * blockDim.x) d[i] = s[i];
}

// ------------------------------------------------------------------ softcap + top-k
// The greedy epilogue needs the winner and the runner-up (near-tie flag); the
// sampled epilogue works on the full host copy of the logits.
constexpr int kTopK = 2;
constexpr int kTkThreads = 256;
static_assert(kTopK <= kTopkRowStride, "a row's candidates fit its output slot");

// Insert (v, i) into a descending list; ties keep the smaller index first.
__device__ __forceinline__ void topk_insert(float (&vals)[kTopK], int (&idx)[kTopK], float v, int i) {
    if (!(v > vals[kTopK - 1] || (v == vals[kTopK - 1] && i < idx[kTopK - 1]))) return;
    int pos = kTopK - 1;
    while (pos > 0 && (v > vals[pos - 1] || (v == vals[pos - 1] && i < idx[pos - 1]))) {
        vals[pos] = vals[pos - 1];
        idx[pos] = idx[pos - 1];
        --pos;
    }
    vals[pos] = v;
    idx[pos] = i;
}

// Stage 1: each block applies the softcap to its slice and emits its top kTopK. Row
// blockIdx.y of a [rows][ld] logits batch; its candidates at part_* + y * gridDim.x * kTopK.
__global__ void softcap_topk_stage1(bf16* logits, int N, float cap, float* part_val, int* part_idx, long long ld) {
    logits += blockIdx.y * ld;
    part_val += static_cast<size_t>(blockIdx.y) * gridDim.x * kTopK;
    part_idx += static_cast<size_t>(blockIdx.y) * gridDim.x * kTopK;
    float vals[kTopK];
    int idx[kTopK];
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
        vals[i] = -FLT_MAX;
        idx[i] = INT32_MAX;
    }
    const float c = rbf(cap);
    for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < N; n += gridDim.x * blockDim.x) {
        float v = bf2f(logits[n]);
        if (cap > 0.f) {
            float d = rbf(v / c);
            float th = rbf(tanhf(d));
            v = rbf(th * c);
            logits[n] = f2bf(v);
        }
        topk_insert(vals, idx, v, n);
    }
    // block merge through shared memory
    __shared__ float sv[kTkThreads * kTopK];
    __shared__ int si[kTkThreads * kTopK];
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
        sv[threadIdx.x * kTopK + i] = vals[i];
        si[threadIdx.x * kTopK + i] = idx[i];
    }
    __syncthreads();
    for (int stride = kTkThreads / 2; stride > 0; stride >>= 1) {
        if (threadIdx.x < stride) {
            const int o = (threadIdx.x + stride) * kTopK;
            for (int i = 0; i < kTopK; ++i) topk_insert(vals, idx, sv[o + i], si[o + i]);
#pragma unroll
            for (int i = 0; i < kTopK; ++i) {
                sv[threadIdx.x * kTopK + i] = vals[i];
                si[threadIdx.x * kTopK + i] = idx[i];
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < kTopK; ++i) {
            part_val[blockIdx.x * kTopK + i] = vals[i];
            part_idx[blockIdx.x * kTopK + i] = idx[i];
        }
    }
}

// Stage 2: one block merges the per-block candidates (strided scan + shared-memory tree).
__global__ void softcap_topk_stage2(const float* part_val, const int* part_idx, int nparts, uint32_t* out_idx,
                                    float* out_val) {
    // one block per row (blockIdx.x); row r's result at out_* + kTopkRowStride r
    part_val += static_cast<size_t>(blockIdx.x) * nparts * kTopK;
    part_idx += static_cast<size_t>(blockIdx.x) * nparts * kTopK;
    out_idx += blockIdx.x * kTopkRowStride;
    out_val += blockIdx.x * kTopkRowStride;
    float vals[kTopK];
    int idx[kTopK];
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
        vals[i] = -FLT_MAX;
        idx[i] = INT32_MAX;
    }
    for (int p = threadIdx.x; p < nparts * kTopK; p += blockDim.x) topk_insert(vals, idx, part_val[p], part_idx[p]);
    __shared__ float sv[kTkThreads * kTopK];
    __shared__ int si[kTkThreads * kTopK];
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
        sv[threadIdx.x * kTopK + i] = vals[i];
        si[threadIdx.x * kTopK + i] = idx[i];
    }
    __syncthreads();
    for (int stride = kTkThreads / 2; stride > 0; stride >>= 1) {
        if (threadIdx.x < stride) {
            const int o = (threadIdx.x + stride) * kTopK;
            for (int i = 0; i < kTopK; ++i) topk_insert(vals, idx, sv[o + i], si[o + i]);
#pragma unroll
            for (int i = 0; i < kTopK; ++i) {
                sv[threadIdx.x * kTopK + i] = vals[i];
                si[threadIdx.x * kTopK + i] = idx[i];
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < kTopK; ++i) {
            out_idx[i] = static_cast<uint32_t>(idx[i]);
            out_val[i] = vals[i];
        }
    }
}

int topk_blocks(int N) { return std::max(1, std::min(num_sms(), (N + kTkThreads - 1) / kTkThreads)); }

}  // namespace

void launch_embed(const uint32_t* ids, int L, const uint32_t* w, const bf16* s, const bf16* b, int H,
                  bf16 embed_scale, bf16* out, cudaStream_t stream) {
    if (H % 64 != 0) throw ArgError("embed: hidden must be a multiple of 64");
    const int words = H / 8;
    dim3 grid((words + 255) / 256, L);
    embed_kernel<<<grid, 256, 0, stream>>>(ids, w, s, b, H, embed_scale, out);
    HYB_LAUNCH_CHECK("embed_kernel");
}

void launch_rms_norm(const bf16* x, const bf16* w, bf16* out, int rows, int D, float eps, cudaStream_t stream) {
    if (rows <= 0) return;
    rms_norm_kernel<<<rows, 256, 0, stream>>>(x, w, out, D, eps);
    HYB_LAUNCH_CHECK("rms_norm_kernel");
}

void launch_resid_norm(const bf16* x, const bf16* post_w, const bf16* resid, const bf16* scalar, bf16* out_h,
                       const bf16* next_w, bf16* out_n, int rows, int D, float eps, cudaStream_t stream) {
    if (rows <= 0) return;
    const bool vec = D % 8 == 0 && D <= 8 * 256 * 4 &&
                     ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(post_w) |
                       reinterpret_cast<uintptr_t>(resid) | reinterpret_cast<uintptr_t>(out_h) |
                       reinterpret_cast<uintptr_t>(next_w) | reinterpret_cast<uintptr_t>(out_n)) & 15u) == 0;
    if (vec) {
        const int c = (D / 8 + 255) / 256;
        switch (c) {
            case 1: resid_norm_vec_kernel<1><<<rows, 256, 0, stream>>>(x, post_w, resid, scalar, out_h, next_w, out_n, D, eps); break;
            case 2: resid_norm_vec_kernel<2><<<rows, 256, 0, stream>>>(x, post_w, resid, scalar, out_h, next_w, out_n, D, eps); break;
            case 3: resid_norm_vec_kernel<3><<<rows, 256, 0, stream>>>(x, post_w, resid, scalar, out_h, next_w, out_n, D, eps); break;
            default: resid_norm_vec_kernel<4><<<rows, 256, 0, stream>>>(x, post_w, resid, scalar, out_h, next_w, out_n, D, eps); break;
        }
        HYB_LAUNCH_CHECK("resid_norm_vec_kernel");
        return;
    }
    const size_t smem = static_cast<size_t>(D) * sizeof(float);
    if (smem > 48 * 1024) throw ArgError("resid_norm: hidden too large");
    resid_norm_kernel<<<rows, 256, smem, stream>>>(x, post_w, resid, scalar, out_h, next_w, out_n, D, eps);
    HYB_LAUNCH_CHECK("resid_norm_kernel");
}

void launch_geglu(const bf16* gate, const bf16* up, bf16* act, int rows, int N, int ld_in, cudaStream_t stream) {
    if (rows <= 0) return;
    dim3 grid(std::min((N + 255) / 256, 64), rows);
    geglu_kernel<<<grid, 256, 0, stream>>>(gate, up, act, N, ld_in);
    HYB_LAUNCH_CHECK("geglu_kernel");
}

void launch_qkv_post(const QkvPostParams& p, cudaStream_t stream) {
    if (p.hd % 64 != 0 || p.hd > 512) throw ArgError("qkv_post: head_dim must be a multiple of 64, <= 512");
    const int warps = p.L * (p.n_heads + 2 * p.n_kv);
    if (warps <= 0) return;
    const int threads = 256;
    const int blocks = (warps * 32 + threads - 1) / threads;
    qkv_post_kernel<<<blocks, threads, 0, stream>>>(p);
    HYB_LAUNCH_CHECK("qkv_post_kernel");
}

void launch_gather_ring(const bf16* cache, int cap, int pos0, int n, int row_elems, bf16* dst,
                        cudaStream_t stream) {
    if (n <= 0) return;
    dim3 grid(std::max(1, std::min((row_elems / 8 + 255) / 256, 8)), n);
    gather_ring_kernel<<<grid, 256, 0, stream>>>(cache, cap, pos0, n, row_elems, dst);
    HYB_LAUNCH_CHECK("gather_ring_kernel");
}

int softcap_topk_scratch_floats(int N) { return topk_blocks(N) * kTopK * 2; }

void launch_softcap_topk(bf16* logits, int N, float cap, float* scratch, int scratch_floats, uint32_t* out_idx,
                         float* out_val, cudaStream_t stream) {
    const int nb = topk_blocks(N);
    if (scratch_floats < nb * kTopK * 2) throw ArgError("softcap_topk: scratch too small");
    float* pv = scratch;
    int* pi = reinterpret_cast<int*>(scratch + nb * kTopK);
    softcap_topk_stage1<<<nb, kTkThreads, 0, stream>>>(logits, N, cap, pv, pi, 0);
    HYB_LAUNCH_CHECK("softcap_topk_stage1");
    softcap_topk_stage2<<<1, kTkThreads, 0, stream>>>(pv, pi, nb, out_idx, out_val);
    HYB_LAUNCH_CHECK("softcap_topk_stage2");
}

void launch_softcap_topk_rows(bf16* logits, int rows, long long ld, int N, float cap, float* scratch,
                              size_t scratch_floats, uint32_t* out_idx, float* out_val, cudaStream_t stream) {
    if (rows <= 0) return;
    const int nb = topk_blocks(N);
    const size_t per = static_cast<size_t>(nb) * kTopK;
    if (scratch_floats < per * 2 * rows) throw ArgError("softcap_topk: scratch too small");
    float* pv = scratch;
    int* pi = reinterpret_cast<int*>(scratch + per * rows);
    softcap_topk_stage1<<<dim3(nb, rows), kTkThreads, 0, stream>>>(logits, N, cap, pv, pi, ld);
    HYB_LAUNCH_CHECK("softcap_topk_stage1");
    softcap_topk_stage2<<<rows, kTkThreads, 0, stream>>>(pv, pi, nb, out_idx, out_val);
    HYB_LAUNCH_CHECK("softcap_topk_stage2");
}

}  // namespace hyb
