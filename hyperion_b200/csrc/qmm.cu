// Prefill affine Q4/g64 GEMM (M >= 2 tokens), legacy tensor-core path.
//
// Replaces mx::quantized_matmul(..., transpose=true, 64, 4, "affine") with M > 1
// (QuantizedLinear::apply, native/hyperion_mlx/src/weights.h:26-37) on the
// prefill path (forward.cc:395-412, 507, 338-343).
//
// Each 128x128 output tile walks K one 64-wide quantization group at a time:
//   * the activation tile [128 x 64] is converted bf16 -> fp16 while staging;
//   * the weight tile [128 rows x 64 codes] is dequantised as
//     w_hat = fp16(s * q + b) (fp32 FMA, one rounding). For codes with
//     b = -8 s the value s * (q - 8) has at most 11 significant bits and is
//     exact in fp16; in general the error is below 2^-12 relative.
//   * fp16 x fp16 -> fp32 mma.sync m16n8k16; bf16 output.
// Global loads for the next group are issued before the current group's MMAs
// (register prefetch into a second shared-memory buffer).
#include "kernels.h"

#include <algorithm>

namespace hyb {
namespace {

constexpr int BM = 128, BN = 128, BK = 64, LDS = BK + 8;  // fp16 elements per smem row
constexpr int kThreads = 256;

__device__ __forceinline__ void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                            const void* p) {
    uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(a));
}

__device__ __forceinline__ uint32_t bf2_to_h2(uint32_t v) {
    float lo = __uint_as_float(v << 16), hi = __uint_as_float(v & 0xFFFF0000u);
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

struct Stage {
    uint4 x[4];       // 32 bf16 of one activation row
    uint4 w;          // 32 codes of one weight row
    uint32_t sb;      // (s, b) bf16 pair
};

__device__ __forceinline__ void load_stage(Stage& st, const bf16* x, const uint32_t* w, const bf16* s,
                                           const bf16* b, int M, int K, int N, int m0, int n0, int grp) {
    const int r = threadIdx.x >> 1, half = threadIdx.x & 1;
    const int m = m0 + r, n = n0 + r;
    const uint4 z = make_uint4(0, 0, 0, 0);
    const uint4* xs = reinterpret_cast<const uint4*>(x + static_cast<size_t>(m) * K + grp * 64 + half * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) st.x[i] = (m < M) ? xs[i] : z;
    const int G = K / 64;
    if (n < N) {
        st.w = ldg_stream(w + static_cast<size_t>(n) * (K / 8) + grp * 8 + half * 4);
        uint32_t sv = __ldg(reinterpret_cast<const uint16_t*>(s) + static_cast<size_t>(n) * G + grp);
        uint32_t bv = __ldg(reinterpret_cast<const uint16_t*>(b) + static_cast<size_t>(n) * G + grp);
        st.sb = sv | (bv << 16);
    } else {
        st.w = z;
        st.sb = 0;
    }
}

__device__ __forceinline__ void store_stage(const Stage& st, __half* As, __half* Bs) {
    const int r = threadIdx.x >> 1, half = threadIdx.x & 1;
    uint32_t* ad = reinterpret_cast<uint32_t*>(As + r * LDS + half * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint4 o;
        o.x = bf2_to_h2(st.x[i].x);
        o.y = bf2_to_h2(st.x[i].y);
        o.z = bf2_to_h2(st.x[i].z);
        o.w = bf2_to_h2(st.x[i].w);
        *reinterpret_cast<uint4*>(ad + 4 * i) = o;
    }
    const float sc = __uint_as_float(st.sb << 16), bi = __uint_as_float(st.sb & 0xFFFF0000u);
    const uint32_t words[4] = {st.w.x, st.w.y, st.w.z, st.w.w};
    uint32_t* bd = reinterpret_cast<uint32_t*>(Bs + r * LDS + half * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float lo = fmaf(sc, static_cast<float>((words[i] >> (8 * j)) & 0xF), bi);
            float hi = fmaf(sc, static_cast<float>((words[i] >> (8 * j + 4)) & 0xF), bi);
            __half2 h = __floats2half2_rn(lo, hi);
            o[j] = *reinterpret_cast<uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(bd + 4 * i) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

__global__ void __launch_bounds__(kThreads, 1)
qmm_mma_kernel(const bf16* __restrict__ x, const uint32_t* __restrict__ w, const bf16* __restrict__ s,
               const bf16* __restrict__ b, bf16* __restrict__ y, int M, int K, int N) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half* As = reinterpret_cast<__half*>(smem_raw);          // [2][BM][LDS]
    __half* Bs = As + 2 * BM * LDS;                            // [2][BN][LDS]
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wm = warp >> 2, wn = warp & 3;  // 2 x 4 warps; warp tile 64 x 32
    const int G = K / 64;

    float acc[4][4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[i][j][c] = 0.f;

    Stage st;
    load_stage(st, x, w, s, b, M, K, N, m0, n0, 0);
    store_stage(st, As, Bs);
    __syncthreads();

    for (int grp = 0; grp < G; ++grp) {
        const int cur = grp & 1;
        if (grp + 1 < G) load_stage(st, x, w, s, b, M, K, N, m0, n0, grp + 1);
        const __half* A = As + cur * BM * LDS;
        const __half* B = Bs + cur * BN * LDS;
#pragma unroll
        for (int kk = 0; kk < BK; kk += 16) {
            uint32_t af[4][4], bfr[4][2];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int row = wm * 64 + i * 16 + (lane & 15);
                const int col = kk + (lane >> 4) * 8;
                ldmatrix_x4(af[i][0], af[i][1], af[i][2], af[i][3], A + row * LDS + col);
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int nrow = wn * 32 + j * 16 + (lane & 7) + ((lane >> 4) << 3);
                const int col = kk + ((lane >> 3) & 1) * 8;
                ldmatrix_x4(bfr[2 * j][0], bfr[2 * j][1], bfr[2 * j + 1][0], bfr[2 * j + 1][1],
                            B + nrow * LDS + col);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    mma_f16_16816(acc[i][j], af[i][0], af[i][1], af[i][2], af[i][3], bfr[j][0], bfr[j][1]);
        }
        if (grp + 1 < G) {
            store_stage(st, As + (cur ^ 1) * BM * LDS, Bs + (cur ^ 1) * BN * LDS);
        }
        __syncthreads();
    }
    // epilogue: bf16 stores
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int col = n0 + wn * 32 + j * 8 + 2 * t;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = m0 + wm * 64 + i * 16 + g + 8 * h;
                if (row < M) {
                    if (col + 1 < N) {
                        __nv_bfloat162 v = __floats2bfloat162_rn(acc[i][j][2 * h], acc[i][j][2 * h + 1]);
                        *reinterpret_cast<__nv_bfloat162*>(y + static_cast<size_t>(row) * N + col) = v;
                    } else if (col < N) {
                        y[static_cast<size_t>(row) * N + col] = f2bf(acc[i][j][2 * h]);
                    }
                }
            }
        }
    }
}

}  // namespace

void launch_qmm(const bf16* x, const uint32_t* w, const bf16* s, const bf16* b, bf16* y, int M, int K,
                int N, cudaStream_t stream) {
    if (K % 64 != 0 || K <= 0 || N <= 0 || M <= 0) throw ArgError("qmm: bad shape");
    const size_t smem = static_cast<size_t>(2 * (BM + BN) * LDS) * sizeof(__half);
    static int attr_dev = -1;
    int dev = 0;
    HYB_CUDA(cudaGetDevice(&dev));
    if (attr_dev != dev) {
        HYB_CUDA(cudaFuncSetAttribute(qmm_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
        attr_dev = dev;
    }
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    qmm_mma_kernel<<<grid, kThreads, smem, stream>>>(x, w, s, b, y, M, K, N);
    HYB_LAUNCH_CHECK("qmm_mma_kernel");
}

void launch_quantized_matmul(const bf16* x, const uint32_t* w, const bf16* s, const bf16* b, bf16* y,
                             int M, int K, int N, cudaStream_t stream) {
    if (M == 1) {
        QmvParams p;
        p.x = x;
        p.w = w;
        p.s = s;
        p.b = b;
        p.y = y;
        p.K = K;
        p.N = N;
        // Programmatic dependent launch: the kernel reads only weights before
        // griddepcontrol.wait, so its first loads may overlap the previous kernel.
        launch_qmv(p, stream, true);
    } else if (qmm_tc_supported(M, K, N)) {
        launch_qmm_tc(x, w, s, b, y, M, K, N, stream);
    } else {
        launch_qmm(x, w, s, b, y, M, K, N, stream);
    }
}

}  // namespace hyb
