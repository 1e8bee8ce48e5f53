// CUDA engine: weight packing, KV state and the forward pass.
//
// Forward semantics follow the reference (paths inside jscott3201/hyperion):
//   decoder layer  forward.cc:510-542     attention  forward.cc:376-508
//   masks/kv_len   forward.cc:46-59, 345-374
//   embed/lm_head  forward.cc:126-160     chunked prefill / decode  model.cc:574-610, 703-718
//   caches         kv_cache.cc:161-347, kv.cc:7-96
#include "engine.h"
#include "safetensors.h"
#include "qmv_pack.cuh"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <mutex>
#include <stdexcept>

namespace hyb {

// ---------------------------------------------------------------- allocation + device info
namespace {
size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

std::atomic<size_t> g_active{0};
std::atomic<size_t> g_peak{0};
std::mutex g_size_mu;
std::vector<std::pair<void*, size_t>> g_sizes;  // small table: pointer -> bytes

void note_alloc(void* p, size_t b) {
    std::lock_guard<std::mutex> lk(g_size_mu);
    g_sizes.emplace_back(p, b);
    size_t now = g_active.fetch_add(b) + b;
    size_t pk = g_peak.load();
    while (now > pk && !g_peak.compare_exchange_weak(pk, now)) {
    }
}
size_t note_free(void* p) {
    std::lock_guard<std::mutex> lk(g_size_mu);
    for (size_t i = 0; i < g_sizes.size(); ++i) {
        if (g_sizes[i].first == p) {
            size_t b = g_sizes[i].second;
            g_sizes[i] = g_sizes.back();
            g_sizes.pop_back();
            g_active.fetch_sub(b);
            return b;
        }
    }
    return 0;
}
}  // namespace

void* dev_alloc(size_t bytes) {
    if (bytes == 0) return nullptr;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        throw std::bad_alloc();
    }
    note_alloc(p, bytes);
    return p;
}
void dev_free(void* p) {
    if (!p) return;
    note_free(p);
    cudaFree(p);
}
size_t dev_active_bytes() { return g_active.load(); }
size_t dev_peak_bytes() { return g_peak.load(); }
void dev_reset_peak() { g_peak.store(g_active.load()); }

int num_sms() {
    static int cached[64] = {0};
    int dev = 0;
    HYB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) dev = 0;
    if (cached[dev] == 0) {
        int n = 0;
        HYB_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        cached[dev] = n;
    }
    return cached[dev];
}

// ---------------------------------------------------------------- synthetic init kernels
//
// Every synthetic value is a pure function of (seed, element key) built from integer
// hashing and IEEE single-rounded float operations only, so a CPU can regenerate the
// exact model (the parity tests rebuild the 12B-shaped weights this way instead of
// shipping gigabytes of checkpoints): codes are the low 32 bits of a SplitMix64 hash,
// normal deviates are looked up in a table of 65536 standard-normal quantiles indexed by
// the top 16 hash bits.
namespace {

constexpr int kNormalTableBits = 16;
constexpr int kNormalTable = 1 << kNormalTableBits;

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ float hash_normal(uint64_t key, const float* __restrict__ ztab) {
    return ztab[mix64(key ^ 0xD1B54A32D192ED03ull) >> (64 - kNormalTableBits)];
}

// Inverse of the standard normal CDF in double precision: Wichura's algorithm AS 241
// (PPND16, Applied Statistics 37:477-484, 1988), relative error about 1e-16.
double normal_quantile(double p) {
    const double q = p - 0.5;
    if (std::fabs(q) <= 0.425) {
        const double r = 0.180625 - q * q;
        const double num = ((((((2509.0809287301226727 * r + 33430.575583588128105) * r + 67265.770927008700853) * r +
                                45921.953931549871457) * r + 13731.693765509461125) * r + 1971.5909503065514427) * r +
                             133.14166789178437745) * r + 3.387132872796366608;
        const double den = ((((((5226.495278852545561 * r + 28729.085735721942674) * r + 39307.89580009271061) * r +
                                21213.794301586595867) * r + 5394.1960214247511077) * r + 687.1870074920579083) * r +
                             42.313330701600911252) * r + 1.0;
        return q * num / den;
    }
    double r = q < 0 ? p : 1.0 - p;
    r = std::sqrt(-std::log(r));
    double v;
    if (r <= 5.0) {
        r -= 1.6;
        v = (((((((7.7454501427834140764e-4 * r + 0.0227238449892691845833) * r + 0.24178072517745061177) * r +
                 1.27045825245236838258) * r + 3.64784832476320460504) * r + 5.7694972214606914055) * r +
              4.6303378461565452959) * r + 1.42343711074968357734) /
            (((((((1.05075007164441684324e-9 * r + 5.475938084995344946e-4) * r + 0.0151986665636164571966) * r +
                 0.14810397642748007459) * r + 0.68976733498510000455) * r + 1.6763848301838038494) * r +
              2.05319162663775882187) * r + 1.0);
    } else {
        r -= 5.0;
        v = (((((((2.01033439929228813265e-7 * r + 2.71155556874348757815e-5) * r + 0.0012426609473880784386) * r +
                 0.026532189526576123093) * r + 0.29656057182850489123) * r + 1.7848265399172913358) * r +
              5.4637849111641143699) * r + 6.6579046435011037772) /
            (((((((2.04426310338993978564e-15 * r + 1.4215117583164458887e-7) * r + 1.8463183175100546818e-5) * r +
                 7.868691311456132591e-4) * r + 0.0148753612908506148525) * r + 0.13692988092273580531) * r +
              0.59983220655588793769) * r + 1.0);
    }
    return q < 0 ? -v : v;
}

// ztab[i] = float(quantile((i + 0.5) / 65536)): a deviate from the top 16 bits of a hash
std::vector<float> normal_table() {
    std::vector<float> t(kNormalTable);
    for (int i = 0; i < kNormalTable; ++i)
        t[i] = static_cast<float>(normal_quantile((i + 0.5) / static_cast<double>(kNormalTable)));
    return t;
}

// A [rows, cols] block of a [*, ld] logical matrix whose element (r, c) is keyed by its
// flat index r * ld + c, so a tensor-parallel shard generates exactly the values of
// the TP = 1 matrix at (row0 + r, col0 + c).
struct Block {
    size_t rows, cols, ld, row0, col0;
    __device__ size_t key(size_t i) const { return (row0 + i / cols) * ld + col0 + i % cols; }
};

__global__ void synth_words_kernel(uint32_t* w, Block blk, uint64_t seed) {
    const size_t n = blk.rows * blk.cols;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        w[i] = static_cast<uint32_t>(mix64(seed * 0x100000001B3ull + blk.key(i)));
}
// scales = bf16(|N(0, std)|), biases = bf16(-8 * scales)
__global__ void synth_sb_kernel(bf16* s, bf16* b, Block blk, uint64_t seed, float std, const float* ztab) {
    const size_t n = blk.rows * blk.cols;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const bf16 sv = f2bf(fabsf(__fmul_rn(std, hash_normal(seed * 0x100000001B3ull + blk.key(i), ztab))));
        s[i] = sv;
        b[i] = f2bf(-8.0f * bf2f(sv));
    }
}
// bf16(mean + std * N(0,1)), multiply and add rounded separately (no contraction)
__global__ void synth_normal_kernel(bf16* x, size_t n, uint64_t seed, float mean, float std, const float* ztab) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        x[i] = f2bf(__fadd_rn(mean, __fmul_rn(std, hash_normal(seed * 0x100000001B3ull + i, ztab))));
}

__global__ void geglu_interleaved_kernel(const bf16* __restrict__ gu, bf16* __restrict__ act, int I) {
    const int l = blockIdx.y;
    const bf16* row = gu + static_cast<size_t>(l) * 2 * I;
    for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < I; n += gridDim.x * blockDim.x) {
        const int base = 32 * (n >> 4) + (n & 15);
        const float g = bf2f(row[base]);
        const float u = bf2f(row[base + 16]);
        const float kC = 0.044677734375f, kK = 0.796875f;
        float x2 = rbf(g * g), x3 = rbf(g * x2);
        float in = rbf(kC * x3);
        in = rbf(in + g);
        in = rbf(kK * in);
        float th = rbf(tanhf(in));
        float ge = rbf(rbf(0.5f * g) * rbf(1.0f + th));
        act[static_cast<size_t>(l) * I + n] = f2bf(ge * u);
    }
}

// (idx0 + vocab0, val0, idx1 + vocab0, val1) of this rank's top-2 as four 32-bit words
__global__ void tp_candidates_kernel(const uint32_t* idx, const float* val, uint32_t vocab0, uint32_t* cand) {
    if (threadIdx.x == 0) {
        cand[0] = idx[0] + vocab0;
        cand[1] = __float_as_uint(val[0]);
        cand[2] = idx[1] + vocab0;
        cand[3] = __float_as_uint(val[1]);
    }
}

// Rows of a batch: (winner, runner-up) of row r with global vocabulary indices at cand + 4 r.
__global__ void tp_candidates_rows_kernel(const uint32_t* idx, const float* val, int rows, uint32_t vocab0,
                                          uint32_t* cand) {
    for (int r = threadIdx.x; r < rows; r += blockDim.x) {
        cand[4 * r + 0] = idx[kTopkRowStride * r] + vocab0;
        cand[4 * r + 1] = __float_as_uint(val[kTopkRowStride * r]);
        cand[4 * r + 2] = idx[kTopkRowStride * r + 1] + vocab0;
        cand[4 * r + 3] = __float_as_uint(val[kTopkRowStride * r + 1]);
    }
}

int grid_for(size_t n) { return static_cast<int>(std::min<size_t>((n + 255) / 256, 4096)); }

// Rows [row0, row0 + rows) x columns [col0, col0 + K) of a synthetic [*, K_full] Q4
// matrix, written at row dst_row of q (whose shape is [q.N, q.K]).
void synth_block(QLin& q, int dst_row, int rows, int row0, int col0, int K_full, uint64_t seed, const float* ztab,
                 cudaStream_t st) {
    const int K = q.K;
    const Block bw{static_cast<size_t>(rows), static_cast<size_t>(K / 8), static_cast<size_t>(K_full / 8),
                   static_cast<size_t>(row0), static_cast<size_t>(col0 / 8)};
    const Block bs{static_cast<size_t>(rows), static_cast<size_t>(K / 64), static_cast<size_t>(K_full / 64),
                   static_cast<size_t>(row0), static_cast<size_t>(col0 / 64)};
    synth_words_kernel<<<grid_for(bw.rows * bw.cols), 256, 0, st>>>(q.w.p + static_cast<size_t>(dst_row) * (K / 8), bw,
                                                                     seed);
    synth_sb_kernel<<<grid_for(bs.rows * bs.cols), 256, 0, st>>>(q.s.p + static_cast<size_t>(dst_row) * (K / 64),
                                                                 q.b.p + static_cast<size_t>(dst_row) * (K / 64), bs,
                                                                 seed ^ 0x5151, 0.02f, ztab);
    HYB_LAUNCH_CHECK("synth_block");
}

void alloc_qlin(QLin& q, int N, int K) {
    q.N = N;
    q.K = K;
    q.w.reset(static_cast<size_t>(N) * K / 8);
    q.s.reset(static_cast<size_t>(N) * K / 64);
    q.b.reset(static_cast<size_t>(N) * K / 64);
}

void synth_qlin(QLin& q, int N, int K, uint64_t seed, const float* ztab, cudaStream_t st) {
    alloc_qlin(q, N, K);
    synth_block(q, 0, N, 0, 0, K, seed, ztab, st);
}

void synth_norm(DevPtr<bf16>& d, size_t n, uint64_t seed, const float* ztab, cudaStream_t st) {
    d.reset(n);
    synth_normal_kernel<<<grid_for(n), 256, 0, st>>>(d.p, n, seed, 1.0f, 0.02f, ztab);
    HYB_LAUNCH_CHECK("synth_norm");
}

// -------- checkpoint helpers
const TensorView& expect(const Checkpoint& ck, const std::string& name, const char* dtype,
                         std::initializer_list<int64_t> shape) {
    const TensorView& t = ck.get(name);
    if (t.dtype != dtype) throw std::runtime_error("tensor " + name + " has dtype " + t.dtype + ", expected " + dtype);
    std::vector<int64_t> want(shape);
    bool ok = t.shape == want;
    if (!ok && want.size() == 1 && want[0] == 1 && t.shape.empty()) ok = true;  // layer_scalar [] or [1]
    if (!ok) throw std::runtime_error("tensor " + name + " has an unexpected shape");
    return t;
}

void upload(void* dst, const TensorView& t) { HYB_CUDA(cudaMemcpy(dst, t.data, t.nbytes, cudaMemcpyHostToDevice)); }

void load_vec(DevPtr<bf16>& d, const Checkpoint& ck, const std::string& name, int64_t n) {
    const TensorView& t = expect(ck, name, "BF16", {n});
    d.reset(static_cast<size_t>(n));
    upload(d.p, t);
}

}  // namespace

// ---------------------------------------------------------------- Model
Model::~Model() {
    if (ws_.h_topk_idx) cudaFreeHost(ws_.h_topk_idx);
    if (ws_.h_topk_val) cudaFreeHost(ws_.h_topk_val);
    if (ws_.h_cand) cudaFreeHost(ws_.h_cand);
    if (ws_.h_ids) cudaFreeHost(ws_.h_ids);
    if (ws_.h_sample) cudaFreeHost(ws_.h_sample);
    if (bws_.h_seqs) cudaFreeHost(bws_.h_seqs);
    if (bws_.h_idx) cudaFreeHost(bws_.h_idx);
    if (bws_.h_val) cudaFreeHost(bws_.h_val);
    if (bws_.h_cand) cudaFreeHost(bws_.h_cand);
    if (stream_) cudaStreamDestroy(stream_);
}

void Model::set_tensor_parallel(int rank, int size, const void* id) {
    if (loaded_) throw ArgError("tensor parallelism must be set before the model is loaded");
    if (size < 1 || rank < 0 || rank >= size) throw ArgError("tensor parallel: bad rank / size");
    tp_rank_ = rank;
    tp_size_ = size;
    if (id) std::memcpy(tp_id_, id, sizeof(tp_id_));
}

void Model::init_common(const Geometry& g) {
    const int T = tp_size_;
    if (T > 1) {
        if (g.n_heads % T || g.intermediate % (16 * T) || g.vocab % (16 * T) || (g.n_heads / T) * g.hd_local % 64 ||
            (g.n_heads / T) * g.hd_global % 64 || (g.intermediate / T) % 64)
            throw ArgError("tensor parallel: heads, MLP rows (16-row tiles, 64-wide groups) and vocabulary "
                           "(16-row blocks) must split evenly over the ranks");
        for (uint32_t i = 0; i < g.n_layers; ++i)
            if (g.n_kv(i) % T) throw ArgError("tensor parallel: KV heads must split evenly over the ranks");
    }
    geo_ = g;
    heads_local_ = static_cast<int>(g.n_heads) / T;
    inter_local_ = static_cast<int>(g.intermediate) / T;
    vocab_local_ = static_cast<int>(g.vocab) / T;
    vocab0_ = tp_rank_ * vocab_local_;
    HYB_CUDA(cudaGetDevice(&device_));
    if (!stream_) HYB_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    auto inv_l = rope_inv_freq(g.hd_local, g.rope_local);
    auto inv_g = rope_inv_freq(g.hd_global, g.rope_global);
    inv_freq_local_.reset(inv_l.size());
    inv_freq_global_.reset(inv_g.size());
    HYB_CUDA(cudaMemcpy(inv_freq_local_.p, inv_l.data(), inv_l.size() * 4, cudaMemcpyHostToDevice));
    HYB_CUDA(cudaMemcpy(inv_freq_global_.p, inv_g.data(), inv_g.size() * 4, cudaMemcpyHostToDevice));
    embed_scale_ = __float2bfloat16_rn(std::sqrt(static_cast<float>(g.hidden)));
    layers_.clear();
    layers_.resize(g.n_layers);
    for (uint32_t i = 0; i < g.n_layers; ++i) {
        LayerW& L = layers_[i];
        L.kind = g.kinds[i];
        L.hd = static_cast<int>(g.head_dim(i));
        L.nkv = static_cast<int>(g.n_kv(i)) / T;
        L.q_rows = heads_local_ * L.hd;
        L.k_rows = L.nkv * L.hd;
        L.v_rows = (L.kind == LayerKind::Full && g.k_eq_v_global) ? 0 : L.nkv * L.hd;
        L.inv_freq = L.kind == LayerKind::Full ? inv_freq_global_.p : inv_freq_local_.p;
    }
}

// Rows [row0, row0 + n) of a packed matrix are themselves a packed matrix of n rows when
// row0 is a multiple of 16: row blocks are independent and their size depends on K only.
MlxView Model::unpack_rows(const unsigned char* packed, int K, int row0, int n, cudaStream_t st) {
    if (row0 % 16) throw std::logic_error("unpack_rows: row0 must start a 16-row block");
    const size_t wb = round_up(static_cast<size_t>(n) * K / 2, 256);
    const size_t sb = round_up(static_cast<size_t>(n) * (K / 64) * 2, 256);
    if (wb + 2 * sb > unpack_.n) throw std::logic_error("unpack_rows: scratch too small");
    const PackGeo pg = pack_geo(K, n);
    MlxView v;
    auto* w = reinterpret_cast<uint32_t*>(unpack_.p);
    auto* sc = reinterpret_cast<bf16*>(unpack_.p + wb);
    auto* bi = reinterpret_cast<bf16*>(unpack_.p + wb + sb);
    launch_qmv_unpack(packed + static_cast<size_t>(row0 / 16) * pg.rb_bytes, K, n, w, sc, bi, st);
    v.w = w;
    v.s = sc;
    v.b = bi;
    return v;
}

void Model::pack_all() {
    auto mlx_bytes = [](int K, int N) {
        return round_up(static_cast<size_t>(N) * K / 2, 256) + 2 * round_up(static_cast<size_t>(N) * (K / 64) * 2, 256);
    };
    size_t scratch = 0;
    auto pack = [&](QLin& q) {
        q.packed.reset(qmv_packed_bytes(q.K, q.N));
        launch_qmv_pack(q.w.p, q.s.p, q.b.p, q.K, q.N, q.packed.p, stream_);
        scratch = std::max(scratch, mlx_bytes(q.K, q.N));
    };
    for (auto& L : layers_) {
        pack(L.qkv);
        pack(L.o);
        pack(L.gateup);
        pack(L.down);
    }
    // the whole embedding table: the embedding gather reads it, and this rank's rows of it
    // (vocab0_ is a multiple of 16) are the tied lm_head
    const int H = embed_.K;
    embed_.packed.reset(qmv_packed_bytes(H, embed_.N));
    launch_qmv_pack(embed_.w.p, embed_.s.p, embed_.b.p, H, embed_.N, embed_.packed.p, stream_);
    lm_packed_ = embed_.packed.p + static_cast<size_t>(vocab0_ / 16) * pack_geo(H, embed_.N).rb_bytes;
    HYB_CUDA(cudaStreamSynchronize(stream_));
    auto drop = [](QLin& q) {
        q.w = DevPtr<uint32_t>();
        q.s = DevPtr<bf16>();
        q.b = DevPtr<bf16>();
    };
    for (auto& L : layers_) {
        drop(L.qkv);
        drop(L.o);
        drop(L.gateup);
        drop(L.down);
    }
    drop(embed_);
    // the lm_head of a batch above the qmv's reach unpacks slices of the same scratch
    const size_t row_bytes = mlx_bytes(H, 16) / 16;
    lm_slice_rows_ = static_cast<int>(std::min<size_t>(vocab_local_, std::max<size_t>(16, scratch / row_bytes / 16 * 16)));
    while (lm_slice_rows_ > 16 && mlx_bytes(H, lm_slice_rows_) > scratch) lm_slice_rows_ -= 16;
    scratch = std::max(scratch, mlx_bytes(H, lm_slice_rows_));
    unpack_.reset(scratch);
}

uint64_t Model::weight_bytes_resident() const {
    uint64_t n = 0;
    auto q = [&](const QLin& x) { n += x.packed.n + x.w.n * 4 + x.s.n * 2 + x.b.n * 2; };
    auto v = [&](const DevPtr<bf16>& x) { n += x.n * 2; };
    for (const auto& L : layers_) {
        q(L.qkv);
        q(L.o);
        q(L.gateup);
        q(L.down);
        v(L.q_norm);
        v(L.k_norm);
        v(L.in_ln);
        v(L.post_attn);
        v(L.pre_ff);
        v(L.post_ff);
        v(L.scalar);
    }
    q(embed_);
    v(final_norm_);
    n += (inv_freq_local_.n + inv_freq_global_.n) * 4;
    return n;
}

uint64_t Model::weight_bytes_algorithmic() const {
    uint64_t n = 0;
    auto q = [&](const QLin& x) { n += static_cast<uint64_t>(x.N) * x.K / 2 + static_cast<uint64_t>(x.N) * (x.K / 64) * 4; };
    for (const auto& L : layers_) {
        q(L.qkv);
        q(L.o);
        q(L.gateup);
        q(L.down);
    }
    q(embed_);
    return n;
}

void Model::load_synthetic(const Geometry& g, uint64_t seed) {
    init_common(g);
    if (tp_size_ > 1) {
        tp_.init(tp_rank_, tp_size_, tp_id_);
        tp_.setup_p2p(g.hidden);  // decode's [hidden] all-reduces go peer to peer
    }
    const int H = static_cast<int>(g.hidden), I = static_cast<int>(g.intermediate);
    const int r = tp_rank_, T = tp_size_;
    const std::vector<float> table = normal_table();
    DevPtr<float> zt(table.size());
    HYB_CUDA(cudaMemcpy(zt.p, table.data(), table.size() * sizeof(float), cudaMemcpyHostToDevice));
    const float* ztab = zt.p;
    uint64_t tag = seed * 1000003ull;
    synth_qlin(embed_, static_cast<int>(g.vocab), H, ++tag, ztab, stream_);  // replicated table
    synth_norm(final_norm_, H, ++tag, ztab, stream_);
    for (auto& L : layers_) {
        // q/k/v: this rank's head rows of the TP = 1 [q; k; v] matrix
        const int qf = static_cast<int>(g.n_heads) * L.hd, kf = L.k_rows * T;
        alloc_qlin(L.qkv, L.q_rows + L.k_rows + L.v_rows, H);
        const uint64_t tq = ++tag;
        synth_block(L.qkv, 0, L.q_rows, r * L.q_rows, 0, H, tq, ztab, stream_);
        synth_block(L.qkv, L.q_rows, L.k_rows, qf + r * L.k_rows, 0, H, tq, ztab, stream_);
        if (L.v_rows)
            synth_block(L.qkv, L.q_rows + L.k_rows, L.v_rows, qf + kf + r * L.v_rows, 0, H, tq, ztab, stream_);
        // o: all rows, this rank's heads' K range
        alloc_qlin(L.o, H, L.q_rows);
        synth_block(L.o, 0, H, 0, r * L.q_rows, qf, ++tag, ztab, stream_);
        // gate/up interleaved by 16-row tiles: this rank's contiguous range of tiles
        alloc_qlin(L.gateup, 2 * inter_local_, H);
        synth_block(L.gateup, 0, 2 * inter_local_, r * 2 * inter_local_, 0, H, ++tag, ztab, stream_);
        // down: all rows, this rank's K range of the MLP
        alloc_qlin(L.down, H, inter_local_);
        synth_block(L.down, 0, H, 0, r * inter_local_, I, ++tag, ztab, stream_);
        synth_norm(L.q_norm, L.hd, ++tag, ztab, stream_);
        synth_norm(L.k_norm, L.hd, ++tag, ztab, stream_);
        synth_norm(L.in_ln, H, ++tag, ztab, stream_);
        synth_norm(L.post_attn, H, ++tag, ztab, stream_);
        synth_norm(L.pre_ff, H, ++tag, ztab, stream_);
        synth_norm(L.post_ff, H, ++tag, ztab, stream_);
        synth_norm(L.scalar, 1, ++tag, ztab, stream_);
    }
    HYB_CUDA(cudaStreamSynchronize(stream_));
    pack_all();
    loaded_ = true;
}

void Model::load_dir(const Geometry& g, const std::string& dir) {
    if (tp_size_ > 1) throw ArgError("tensor-parallel loading from a checkpoint directory is not supported yet");
    Checkpoint ck(dir);
    init_common(g);
    const int64_t H = g.hidden, I = g.intermediate, V = g.vocab;
    const std::string pre = "language_model.model.";
    // tied embedding / lm_head table
    {
        const auto& w = expect(ck, pre + "embed_tokens.weight", "U32", {V, H / 8});
        const auto& s = expect(ck, pre + "embed_tokens.scales", "BF16", {V, H / 64});
        const auto& b = expect(ck, pre + "embed_tokens.biases", "BF16", {V, H / 64});
        embed_.N = static_cast<int>(V);
        embed_.K = static_cast<int>(H);
        embed_.w.reset(w.nbytes / 4);
        embed_.s.reset(s.nbytes / 2);
        embed_.b.reset(b.nbytes / 2);
        upload(embed_.w.p, w);
        upload(embed_.s.p, s);
        upload(embed_.b.p, b);
    }
    load_vec(final_norm_, ck, pre + "norm.weight", H);
    for (uint32_t i = 0; i < g.n_layers; ++i) {
        LayerW& L = layers_[i];
        const std::string p = pre + "layers." + std::to_string(i) + ".";
        const std::string a = p + "self_attn.";
        const bool has_v = ck.has(a + "v_proj.weight");
        const bool schema_sliding = has_v;
        if ((schema_sliding ? LayerKind::Sliding : LayerKind::Full) != L.kind) {
            throw std::runtime_error("layer " + std::to_string(i) + " weight schema (" +
                                     (schema_sliding ? "sliding" : "global") +
                                     ") disagrees with geometry layer_types");
        }
        if (!has_v) L.v_rows = 0;
        const int64_t qkv_rows = L.q_rows + L.k_rows + L.v_rows;
        L.qkv.N = static_cast<int>(qkv_rows);
        L.qkv.K = static_cast<int>(H);
        L.qkv.w.reset(static_cast<size_t>(qkv_rows) * H / 8);
        L.qkv.s.reset(static_cast<size_t>(qkv_rows) * H / 64);
        L.qkv.b.reset(static_cast<size_t>(qkv_rows) * H / 64);
        int64_t row = 0;
        auto put = [&](const std::string& base, int64_t rows) {
            const auto& w = expect(ck, base + ".weight", "U32", {rows, H / 8});
            const auto& s = expect(ck, base + ".scales", "BF16", {rows, H / 64});
            const auto& b = expect(ck, base + ".biases", "BF16", {rows, H / 64});
            upload(L.qkv.w.p + row * (H / 8), w);
            upload(L.qkv.s.p + row * (H / 64), s);
            upload(L.qkv.b.p + row * (H / 64), b);
            row += rows;
        };
        put(a + "q_proj", L.q_rows);
        put(a + "k_proj", L.k_rows);
        if (has_v) put(a + "v_proj", L.v_rows);
        {
            const int64_t K = static_cast<int64_t>(g.n_heads) * L.hd;
            const auto& w = expect(ck, a + "o_proj.weight", "U32", {H, K / 8});
            const auto& s = expect(ck, a + "o_proj.scales", "BF16", {H, K / 64});
            const auto& b = expect(ck, a + "o_proj.biases", "BF16", {H, K / 64});
            L.o.N = static_cast<int>(H);
            L.o.K = static_cast<int>(K);
            L.o.w.reset(w.nbytes / 4);
            L.o.s.reset(s.nbytes / 2);
            L.o.b.reset(b.nbytes / 2);
            upload(L.o.w.p, w);
            upload(L.o.s.p, s);
            upload(L.o.b.p, b);
        }
        {
            // gate/up interleaved by 16-row tiles: tile 2t = gate rows [16t, 16t+16), 2t+1 = up rows
            const auto& gw = expect(ck, p + "mlp.gate_proj.weight", "U32", {I, H / 8});
            const auto& gs = expect(ck, p + "mlp.gate_proj.scales", "BF16", {I, H / 64});
            const auto& gb = expect(ck, p + "mlp.gate_proj.biases", "BF16", {I, H / 64});
            const auto& uw = expect(ck, p + "mlp.up_proj.weight", "U32", {I, H / 8});
            const auto& us = expect(ck, p + "mlp.up_proj.scales", "BF16", {I, H / 64});
            const auto& ub = expect(ck, p + "mlp.up_proj.biases", "BF16", {I, H / 64});
            L.gateup.N = static_cast<int>(2 * I);
            L.gateup.K = static_cast<int>(H);
            L.gateup.w.reset(static_cast<size_t>(2 * I) * H / 8);
            L.gateup.s.reset(static_cast<size_t>(2 * I) * H / 64);
            L.gateup.b.reset(static_cast<size_t>(2 * I) * H / 64);
            auto inter = [&](void* dst, const TensorView& src, size_t row_bytes, int which) {
                HYB_CUDA(cudaMemcpy2D(static_cast<char*>(dst) + which * 16 * row_bytes, 32 * row_bytes, src.data,
                                      16 * row_bytes, 16 * row_bytes, static_cast<size_t>(I / 16),
                                      cudaMemcpyHostToDevice));
            };
            inter(L.gateup.w.p, gw, H / 2, 0);
            inter(L.gateup.w.p, uw, H / 2, 1);
            inter(L.gateup.s.p, gs, H / 64 * 2, 0);
            inter(L.gateup.s.p, us, H / 64 * 2, 1);
            inter(L.gateup.b.p, gb, H / 64 * 2, 0);
            inter(L.gateup.b.p, ub, H / 64 * 2, 1);
        }
        {
            const auto& w = expect(ck, p + "mlp.down_proj.weight", "U32", {H, I / 8});
            const auto& s = expect(ck, p + "mlp.down_proj.scales", "BF16", {H, I / 64});
            const auto& b = expect(ck, p + "mlp.down_proj.biases", "BF16", {H, I / 64});
            L.down.N = static_cast<int>(H);
            L.down.K = static_cast<int>(I);
            L.down.w.reset(w.nbytes / 4);
            L.down.s.reset(s.nbytes / 2);
            L.down.b.reset(b.nbytes / 2);
            upload(L.down.w.p, w);
            upload(L.down.s.p, s);
            upload(L.down.b.p, b);
        }
        load_vec(L.q_norm, ck, a + "q_norm.weight", L.hd);
        load_vec(L.k_norm, ck, a + "k_norm.weight", L.hd);
        load_vec(L.in_ln, ck, p + "input_layernorm.weight", H);
        load_vec(L.post_attn, ck, p + "post_attention_layernorm.weight", H);
        load_vec(L.pre_ff, ck, p + "pre_feedforward_layernorm.weight", H);
        load_vec(L.post_ff, ck, p + "post_feedforward_layernorm.weight", H);
        {
            const TensorView& t = expect(ck, p + "layer_scalar", "BF16", {1});
            L.scalar.reset(1);
            HYB_CUDA(cudaMemcpy(L.scalar.p, t.data, 2, cudaMemcpyHostToDevice));
        }
    }
    pack_all();
    loaded_ = true;
}

std::unique_ptr<KvState> Model::new_kv() const {
    auto kv = std::make_unique<KvState>();
    const uint32_t cap = geo_.window + 8;  // window + gamma_max (kv_cache.h:16, kv.cc:233-235)
    size_t total = 0;
    for (const auto& L : layers_)
        if (L.kind == LayerKind::Sliding) total += 2 * static_cast<size_t>(cap) * L.nkv * L.hd;
    if (total) {
        kv->ring_arena.reset(total);
        HYB_CUDA(cudaMemsetAsync(kv->ring_arena.p, 0, total * 2, stream_));
    }
    size_t at = 0;
    for (const auto& L : layers_) {
        if (L.kind == LayerKind::Sliding) {
            LocalCache c;
            c.nkv = L.nkv;
            c.hd = L.hd;
            c.cap = cap;
            const size_t n = static_cast<size_t>(c.cap) * c.nkv * c.hd;
            c.k = kv->ring_arena.p + at;
            c.v = c.k + n;
            at += 2 * n;
            encode_kv_tensor_map(&c.tk, c.k, static_cast<int>(c.cap), c.nkv, c.hd);
            encode_kv_tensor_map(&c.tv, c.v, static_cast<int>(c.cap), c.nkv, c.hd);
            kv->local.push_back(c);
        } else {
            GlobalCache c;
            c.nkv = L.nkv;
            c.hd = L.hd;
            kv->global.push_back(c);
        }
    }
    HYB_CUDA(cudaStreamSynchronize(stream_));
    return kv;
}

std::unique_ptr<KvState> Model::clone_kv(const KvState& src, uint32_t last_token) const {
    auto kv = std::make_unique<KvState>();
    kv->local = src.local;
    kv->global = src.global;
    // the same layout in new arenas: every pointer moves by the arenas' distance
    if (src.ring_arena.n) {
        kv->ring_arena.reset(src.ring_arena.n);
        HYB_CUDA(cudaMemcpyAsync(kv->ring_arena.p, src.ring_arena.p, src.ring_arena.n * 2, cudaMemcpyDeviceToDevice,
                                 stream_));
        for (auto& c : kv->local) {
            c.k = kv->ring_arena.p + (c.k - src.ring_arena.p);
            c.v = kv->ring_arena.p + (c.v - src.ring_arena.p);
            encode_kv_tensor_map(&c.tk, c.k, static_cast<int>(c.cap), c.nkv, c.hd);
            encode_kv_tensor_map(&c.tv, c.v, static_cast<int>(c.cap), c.nkv, c.hd);
        }
    }
    if (src.global_arena.n) {
        kv->global_arena.reset(src.global_arena.n);
        HYB_CUDA(cudaMemcpyAsync(kv->global_arena.p, src.global_arena.p, src.global_arena.n * 2,
                                 cudaMemcpyDeviceToDevice, stream_));
        for (auto& c : kv->global) {
            if (c.capacity == 0) continue;
            c.k = kv->global_arena.p + (c.k - src.global_arena.p);
            c.v = kv->global_arena.p + (c.v - src.global_arena.p);
            encode_kv_tensor_map(&c.tk, c.k, static_cast<int>(c.capacity), c.nkv, c.hd);
            encode_kv_tensor_map(&c.tv, c.v, static_cast<int>(c.capacity), c.nkv, c.hd);
        }
    }
    kv->offset = src.offset;
    kv->last_token = last_token;
    HYB_CUDA(cudaStreamSynchronize(stream_));
    return kv;
}

bool Model::grow_globals(KvState& kv, uint32_t n_tokens, DevPtr<bf16>* old) const {
    std::vector<uint32_t> caps(kv.global.size());
    bool grows = false;
    size_t total = 0;
    for (size_t i = 0; i < kv.global.size(); ++i) {
        const GlobalCache& c = kv.global[i];
        const uint64_t need = (static_cast<uint64_t>(c.committed) + n_tokens + 255) / 256 * 256;
        if (need > 0xFFFFFFFFull) throw std::overflow_error("KV operation exceeds representable cache dimensions");
        if (need > c.capacity) grows = true;
        caps[i] = static_cast<uint32_t>(std::max<uint64_t>(need, c.capacity));
        total += 2 * static_cast<size_t>(caps[i]) * c.nkv * c.hd;
    }
    if (!grows) return false;
    DevPtr<bf16> arena(total);
    HYB_CUDA(cudaMemsetAsync(arena.p, 0, total * 2, stream_));
    size_t at = 0;
    for (size_t i = 0; i < kv.global.size(); ++i) {
        GlobalCache& c = kv.global[i];
        const size_t row = static_cast<size_t>(c.nkv) * c.hd;
        bf16* nk = arena.p + at;
        bf16* nv = nk + caps[i] * row;
        at += 2 * caps[i] * row;
        if (c.capacity > 0) {
            HYB_CUDA(cudaMemcpyAsync(nk, c.k, c.capacity * row * 2, cudaMemcpyDeviceToDevice, stream_));
            HYB_CUDA(cudaMemcpyAsync(nv, c.v, c.capacity * row * 2, cudaMemcpyDeviceToDevice, stream_));
        }
        c.k = nk;
        c.v = nv;
        c.capacity = caps[i];
        encode_kv_tensor_map(&c.tk, c.k, static_cast<int>(c.capacity), c.nkv, c.hd);
        encode_kv_tensor_map(&c.tv, c.v, static_cast<int>(c.capacity), c.nkv, c.hd);
    }
    HYB_CUDA(cudaStreamSynchronize(stream_));
    *old = std::move(kv.global_arena);
    kv.global_arena = std::move(arena);
    return true;
}

void Model::reserve(KvState& kv, uint32_t n_tokens) const {
    DevPtr<bf16> old;
    grow_globals(kv, n_tokens, &old);  // the old arena is freed here, after the copies
}

bool Model::predict_call_bytes(const KvState& kv, uint32_t n_tokens, uint64_t* bytes) const {
    uint64_t b = 0, arena = 0;
    bool grows = false;
    for (const auto& c : kv.global) {
        const uint64_t need = (static_cast<uint64_t>(c.committed) + n_tokens + 255) / 256 * 256;
        if (need > 0xFFFFFFFFull) return false;
        if (need > c.capacity) grows = true;
        arena += std::max<uint64_t>(need, c.capacity) * c.nkv * c.hd * 2 * 2;
    }
    if (grows) b += arena;  // the staged arena holds every global cache
    for (const auto& c : kv.local)
        if (static_cast<uint64_t>(c.committed) + n_tokens > 0xFFFFFFFFull) return false;
    if (grows && n_tokens > static_cast<uint32_t>(kSpecMax) && kv.offset > 0) b += kv.ring_arena.n * 2;
    // workspace the call would newly allocate (ensure_workspace): a prefill runs chunks of
    // up to 2048 rows, decode one row per forward
    const Geometry& g = geo_;
    const bool prefill = kv.offset == 0;
    const uint64_t rows = prefill ? std::min<uint32_t>(n_tokens, 2048) : 1;
    if (rows > static_cast<uint64_t>(ws_.chunk_cap)) {
        uint64_t max_qkv = 0, max_attn = 0, max_kv_row = 0;
        for (const auto& L : layers_) {
            max_qkv = std::max<uint64_t>(max_qkv, L.q_rows + L.k_rows + L.v_rows);
            max_attn = std::max<uint64_t>(max_attn, L.q_rows);
            max_kv_row = std::max<uint64_t>(max_kv_row, static_cast<uint64_t>(L.nkv) * L.hd);
        }
        const uint64_t H = g.hidden, I = static_cast<uint64_t>(inter_local_);
        b += 2 * rows * (6 * H + max_qkv + 2 * max_attn + 3 * I) + 4 * rows + 2 * 2 * (rows + g.window) * max_kv_row;
    }
    const uint64_t keys = std::min<uint64_t>(static_cast<uint64_t>(kv.offset) + n_tokens, 32768);
    size_t need = 0;
    for (const auto& L : layers_)
        need = std::max(need, decode_attn_scratch_bytes(heads_local_, L.nkv, L.hd, static_cast<int>(keys)));
    if (need > ws_.attn_scratch_bytes) b += std::max(need, ws_.attn_scratch_bytes * 2);
    *bytes = b;
    return true;
}

KvTransaction Model::begin_kv_transaction(KvState& kv, uint32_t n_tokens) const {
    KvTransaction t;
    bool grows = false;
    for (const auto& c : kv.global)
        if ((static_cast<uint64_t>(c.committed) + n_tokens + 255) / 256 * 256 > c.capacity) grows = true;
    if (!grows) return t;
    t.active = true;
    t.offset = kv.offset;
    t.last_token = kv.last_token;
    for (const auto& c : kv.local) t.local_committed.push_back(c.committed);
    for (const auto& c : kv.global) {
        t.global_committed.push_back(c.committed);
        KvTransaction::Global gk;
        gk.k = c.k;
        gk.v = c.v;
        gk.capacity = c.capacity;
        gk.tk = c.tk;
        gk.tv = c.tv;
        t.globals.push_back(gk);
    }
    if (n_tokens > static_cast<uint32_t>(kSpecMax) && kv.offset > 0 && kv.ring_arena.n) {
        t.ring_backup.reset(kv.ring_arena.n);
        HYB_CUDA(cudaMemcpyAsync(t.ring_backup.p, kv.ring_arena.p, kv.ring_arena.n * 2, cudaMemcpyDeviceToDevice,
                                 stream_));
    }
    grow_globals(kv, n_tokens, &t.global_arena);  // synchronises the stream
    return t;
}

void Model::rollback_kv_transaction(KvState& kv, KvTransaction& t) const {
    if (!t.active) return;
    // work of the failed call may still be queued: let it finish before buffers change hands
    cudaError_t e = cudaStreamSynchronize(stream_);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        kv.poisoned = true;  // the device is in an error state: the cache contents are unknown
        return;
    }
    for (size_t i = 0; i < t.globals.size(); ++i) {
        GlobalCache& c = kv.global[i];
        c.k = t.globals[i].k;
        c.v = t.globals[i].v;
        c.capacity = t.globals[i].capacity;
        c.tk = t.globals[i].tk;
        c.tv = t.globals[i].tv;
    }
    kv.global_arena = std::move(t.global_arena);
    if (t.ring_backup.n)
        HYB_CUDA(cudaMemcpyAsync(kv.ring_arena.p, t.ring_backup.p, t.ring_backup.n * 2, cudaMemcpyDeviceToDevice,
                                 stream_));
    for (size_t i = 0; i < kv.local.size(); ++i) kv.local[i].committed = t.local_committed[i];
    for (size_t i = 0; i < kv.global.size(); ++i) kv.global[i].committed = t.global_committed[i];
    kv.offset = t.offset;
    kv.last_token = t.last_token;
    HYB_CUDA(cudaStreamSynchronize(stream_));
    t = KvTransaction{};
}

uint64_t Model::local_kv_bytes(const KvState& kv) const {
    uint64_t b = 0;
    for (const auto& c : kv.local) b += static_cast<uint64_t>(c.cap) * c.nkv * c.hd * 2 * 2;
    return b;
}
uint64_t Model::global_kv_bytes(const KvState& kv) const {
    uint64_t b = 0;
    for (const auto& c : kv.global) b += static_cast<uint64_t>(c.capacity) * c.nkv * c.hd * 2 * 2;
    return b;
}

void Model::ensure_workspace(int tokens, uint32_t max_keys) {
    const Geometry& g = geo_;
    const int H = static_cast<int>(g.hidden), I = inter_local_;
    int max_qkv = 0, max_attn = 0, max_kv_row = 0, max_hd = 0;
    for (const auto& L : layers_) {
        max_qkv = std::max(max_qkv, L.q_rows + L.k_rows + L.v_rows);
        max_attn = std::max(max_attn, L.q_rows);
        max_kv_row = std::max(max_kv_row, L.nkv * L.hd);
        max_hd = std::max(max_hd, L.hd);
    }
    if (tokens > ws_.chunk_cap) {
        const size_t C = static_cast<size_t>(tokens);
        ws_.h_a.reset(C * H);
        ws_.h_b.reset(C * H);
        ws_.h_e.reset(C * H);
        ws_.xn.reset(C * H);
        ws_.qkv.reset(C * max_qkv);
        ws_.q.reset(C * max_attn);
        ws_.attn.reset(C * max_attn);
        ws_.o.reset(C * H);
        ws_.gu.reset(C * 2 * I);
        ws_.act.reset(C * I);
        ws_.dn.reset(C * H);
        ws_.ids.reset(C);
        // keys of one attention call: trailing window prefix + chunk (local) or the
        // chunk itself at offset 0
        const size_t kv_rows = C + g.window;
        ws_.kbuf.reset(kv_rows * max_kv_row);
        ws_.vbuf.reset(kv_rows * max_kv_row);
        ws_.chunk_cap = tokens;
        if (ws_.h_ids) cudaFreeHost(ws_.h_ids);
        HYB_CUDA(cudaMallocHost(&ws_.h_ids, C * sizeof(uint32_t)));
        ws_.h_ids_cap = tokens;
    }
    if (ws_.logits.n == 0) {
        ws_.logits.reset(vocab_local_);
        if (tp_size_ > 1) {
            ws_.cand.reset(static_cast<size_t>(4) * tp_size_ * 2);  // [own 4][gathered TP x 4]
            ws_.logits_all.reset(g.vocab);
        }
        const int tsf = softcap_topk_scratch_floats(vocab_local_);
        ws_.topk_scratch.reset(tsf);
        ws_.topk_idx.reset(8);
        ws_.topk_val.reset(8);
        HYB_CUDA(cudaMallocHost(&ws_.h_topk_idx, 8 * sizeof(uint32_t)));
        HYB_CUDA(cudaMallocHost(&ws_.h_topk_val, 8 * sizeof(float)));
        HYB_CUDA(cudaMallocHost(&ws_.h_cand, static_cast<size_t>(4) * tp_size_ * sizeof(uint32_t)));
    }
    size_t need = 0;
    for (const auto& L : layers_)
        need = std::max(need, decode_attn_scratch_bytes(heads_local_, L.nkv, L.hd,
                                                        static_cast<int>(std::max<uint32_t>(max_keys, 1))));
    if (need > ws_.attn_scratch_bytes) {
        // grow geometrically so decode does not reallocate every 256 tokens
        size_t target = std::max(need, ws_.attn_scratch_bytes * 2);
        ws_.attn_scratch.reset(target);
        HYB_CUDA(cudaMemsetAsync(ws_.attn_scratch.p, 0, target, stream_));
        ws_.attn_scratch_bytes = target;
    }
}

void Model::forward_chunk(KvState& kv, int L, uint32_t offset) {
    const Geometry& g = geo_;
    const int H = static_cast<int>(g.hidden), I = inter_local_;
    const int nh = heads_local_;
    cudaStream_t st = stream_;
    bf16* h_cur = ws_.h_a.p;
    bf16* h_alt = ws_.h_b.p;
    // y[L, q.N] = x[L, q.K] · qᵀ through the tcgen05 GEMM over the MLX layout, re-derived
    // from the packed copy per projection
    auto gemm = [&](const bf16* x, const QLin& q, bf16* y) {
        const MlxView m = unpack_rows(q.packed.p, q.K, 0, q.N, st);
        launch_quantized_matmul(x, m.w, m.s, m.b, y, L, q.K, q.N, st);
    };
    launch_embed_packed(ws_.ids.p, L, embed_.packed.p, H, embed_.N, embed_scale_, h_cur, st);
    launch_rms_norm(h_cur, layers_[0].in_ln.p, ws_.xn.p, L, H, g.eps, st);
    size_t li = 0, gi = 0;
    for (uint32_t layer = 0; layer < g.n_layers; ++layer) {
        LayerW& W = layers_[layer];
        const int hd = W.hd, nkv = W.nkv;
        const int qkv_ld = W.q_rows + W.k_rows + W.v_rows;
        gemm(ws_.xn.p, W.qkv, ws_.qkv.p);
        const uint32_t committed = offset + static_cast<uint32_t>(L);
        QkvPostParams qp;
        qp.qkv = ws_.qkv.p;
        qp.L = L;
        qp.ld = qkv_ld;
        qp.n_heads = nh;
        qp.n_kv = nkv;
        qp.hd = hd;
        qp.v_from_k = W.v_rows == 0;
        qp.q_norm = W.q_norm.p;
        qp.k_norm = W.k_norm.p;
        qp.inv_freq = W.inv_freq;
        qp.pos0 = static_cast<int>(offset);
        qp.eps = g.eps;
        qp.q_out = ws_.q.p;
        PrefillAttnParams ap;
        ap.q = ws_.q.p;
        ap.out = ws_.attn.p;
        ap.Lq = L;
        ap.n_heads = nh;
        ap.n_kv = nkv;
        ap.hd = hd;
        ap.q_pos0 = static_cast<int>(offset);
        ap.scale = 1.0f;
        ap.rounding = attn_rounding_;
        const size_t row = static_cast<size_t>(nkv) * hd;
        if (W.kind == LayerKind::Sliding) {
            LocalCache& c = kv.local[li++];
            // continuation: gather the committed trailing window BEFORE the append
            // (forward.cc:444-457); the chunk's own K/V follow it contiguously
            const uint32_t pre = offset > 0 ? std::min(g.window, offset) : 0;
            if (pre > 0) {
                launch_gather_ring(c.k, static_cast<int>(c.cap), static_cast<int>(offset - pre), static_cast<int>(pre),
                                   static_cast<int>(row), ws_.kbuf.p, st);
                launch_gather_ring(c.v, static_cast<int>(c.cap), static_cast<int>(offset - pre), static_cast<int>(pre),
                                   static_cast<int>(row), ws_.vbuf.p, st);
            }
            qp.k_out = ws_.kbuf.p + pre * row;
            qp.v_out = ws_.vbuf.p + pre * row;
            qp.k_cache = c.k;
            qp.v_cache = c.v;
            qp.cache_cap = static_cast<int>(c.cap);
            // a chunk longer than the ring leaves only its last `cap` tokens resident
            qp.cache_first = std::max(0, L - static_cast<int>(c.cap));
            launch_qkv_post(qp, st);
            c.committed = committed;
            ap.k = ws_.kbuf.p;
            ap.v = ws_.vbuf.p;
            ap.Lk = static_cast<int>(pre) + L;
            ap.k_pos0 = static_cast<int>(offset - pre);
            ap.window = static_cast<int>(g.window);
        } else {
            GlobalCache& c = kv.global[gi++];
            if (c.capacity < committed) throw std::runtime_error("global cache not reserved");
            qp.k_cache = c.k;
            qp.v_cache = c.v;
            qp.cache_cap = static_cast<int>(c.capacity);
            qp.cache_first = 0;
            launch_qkv_post(qp, st);
            c.committed = committed;
            ap.k = c.k;
            ap.v = c.v;
            ap.Lk = static_cast<int>(committed);
            ap.k_pos0 = 0;
            ap.window = 0;
        }
        launch_prefill_attn(ap, st);
        gemm(ws_.attn.p, W.o, ws_.o.p);
        tp_.all_reduce_sum_bf16(ws_.o.p, static_cast<size_t>(L) * H, st);  // row-parallel o_proj
        launch_resid_norm(ws_.o.p, W.post_attn.p, h_cur, nullptr, h_alt, W.pre_ff.p, ws_.xn.p, L, H, g.eps, st);
        if (qmm_tc_geglu_supported(L, H, W.gateup.N)) {
            // GeGLU in the GEMM's epilogue: the interleaved gate/up output never reaches memory
            const MlxView m = unpack_rows(W.gateup.packed.p, H, 0, W.gateup.N, st);
            launch_qmm_tc(ws_.xn.p, m.w, m.s, m.b, ws_.act.p, L, H, W.gateup.N, st, true);
        } else {
            gemm(ws_.xn.p, W.gateup, ws_.gu.p);
            dim3 grid(std::min((I + 255) / 256, 64), L);
            geglu_interleaved_kernel<<<grid, 256, 0, st>>>(ws_.gu.p, ws_.act.p, I);
            HYB_LAUNCH_CHECK("geglu_interleaved_kernel");
        }
        gemm(ws_.act.p, W.down, ws_.dn.p);
        tp_.all_reduce_sum_bf16(ws_.dn.p, static_cast<size_t>(L) * H, st);  // row-parallel down_proj
        const bf16* next_w = (layer + 1 < g.n_layers) ? layers_[layer + 1].in_ln.p : final_norm_.p;
        launch_resid_norm(ws_.dn.p, W.post_ff.p, h_alt, W.scalar.p, h_cur, next_w, ws_.xn.p, L, H, g.eps, st);
    }
}

StepOut Model::epilogue(const bf16* final_row, bool fused_prologue, const bf16* dn, const bf16* resid,
                        std::vector<uint16_t>* logits_out, const SampleSpec* sample) {
    const Geometry& g = geo_;
    const int H = static_cast<int>(g.hidden);
    QmvParams p;  // lm_head over this rank's vocabulary rows (all of them when TP = 1)
    p.packed = lm_packed_;
    p.y = ws_.logits.p;
    p.K = H;
    p.N = vocab_local_;
    p.eps = g.eps;
    if (fused_prologue) {
        const LayerW& last = layers_.back();
        p.prologue = QmvPrologue::kResidNorm;
        p.x = dn;
        p.resid = resid;
        p.post_w = last.post_ff.p;
        p.scalar = last.scalar.p;
        p.norm_w = final_norm_.p;
        p.h_out = ws_.h_a.p;
        if (tp_.active() && tp_.fused_ready()) {  // the last down_proj's all-reduce
            p.ar_mode = 2;
            p.ar = last_ar_;
        }
    } else {
        p.x = final_row;
    }
    launch_qmv(p, stream_, fused_prologue);
    launch_softcap_topk(ws_.logits.p, vocab_local_, g.softcap, ws_.topk_scratch.p,
                        static_cast<int>(ws_.topk_scratch.n), ws_.topk_idx.p, ws_.topk_val.p, stream_);
    const int T = tp_size_;
    if (sample) {
        // the sampler reads the whole post-softcap row: with tensor parallelism every rank
        // gathers it and samples the same bits (same row, same seed)
        const bf16* row = ws_.logits.p;
        if (T > 1) {
            tp_.all_gather_bytes(ws_.logits.p, ws_.logits_all.p, static_cast<size_t>(vocab_local_) * 2, stream_);
            row = ws_.logits_all.p;
        }
        if (ws_.sample.n == 0) {
            ws_.sample.reset(sizeof(SampleResult));
            HYB_CUDA(cudaMallocHost(&ws_.h_sample, sizeof(SampleResult)));
        }
        SampleResult* d = reinterpret_cast<SampleResult*>(ws_.sample.p);
        launch_sample(row, static_cast<int>(g.vocab), *sample, d, stream_);
        HYB_CUDA(cudaMemcpyAsync(ws_.h_sample, d, sizeof(SampleResult), cudaMemcpyDeviceToHost, stream_));
        if (logits_out) {
            logits_out->resize(g.vocab);
            HYB_CUDA(cudaMemcpyAsync(logits_out->data(), row, static_cast<size_t>(g.vocab) * 2, cudaMemcpyDeviceToHost,
                                     stream_));
        }
        HYB_CUDA(cudaStreamSynchronize(stream_));
        if (T > 1 && tp_.take_wait_errors(stream_))
            throw CudaError("tensor-parallel all-reduce: a wait for a peer's flag gave up");
        const SampleResult& r = *ws_.h_sample;
        StepOut out;
        out.token = r.token;
        out.logit = r.logit;
        out.near_tie = false;  // sampled steps report no near-tie events (forward.cc:191-322)
        for (uint32_t i = 0; i < 8; ++i) {
            out.topk_idx[i] = r.topk_idx[i];
            out.topk_val[i] = r.topk_val[i];
        }
        return out;
    }
    if (T > 1) {
        // every rank's (winner, runner-up) with global vocabulary indices, all-gathered
        tp_candidates_kernel<<<1, 32, 0, stream_>>>(ws_.topk_idx.p, ws_.topk_val.p, static_cast<uint32_t>(vocab0_),
                                                   ws_.cand.p);
        HYB_LAUNCH_CHECK("tp_candidates_kernel");
        tp_.all_gather_bytes(ws_.cand.p, ws_.cand.p + 4, 16, stream_);
        HYB_CUDA(cudaMemcpyAsync(ws_.h_cand, ws_.cand.p + 4, static_cast<size_t>(T) * 16, cudaMemcpyDeviceToHost,
                                 stream_));
        if (logits_out) {
            tp_.all_gather_bytes(ws_.logits.p, ws_.logits_all.p, static_cast<size_t>(vocab_local_) * 2, stream_);
            logits_out->resize(g.vocab);
            HYB_CUDA(cudaMemcpyAsync(logits_out->data(), ws_.logits_all.p, static_cast<size_t>(g.vocab) * 2,
                                     cudaMemcpyDeviceToHost, stream_));
        }
    } else {
        HYB_CUDA(cudaMemcpyAsync(ws_.h_topk_idx, ws_.topk_idx.p, 8 * sizeof(uint32_t), cudaMemcpyDeviceToHost, stream_));
        HYB_CUDA(cudaMemcpyAsync(ws_.h_topk_val, ws_.topk_val.p, 8 * sizeof(float), cudaMemcpyDeviceToHost, stream_));
        if (logits_out) {
            logits_out->resize(g.vocab);
            HYB_CUDA(cudaMemcpyAsync(logits_out->data(), ws_.logits.p, static_cast<size_t>(g.vocab) * 2,
                                     cudaMemcpyDeviceToHost, stream_));
        }
    }
    HYB_CUDA(cudaStreamSynchronize(stream_));
    if (T > 1 && tp_.take_wait_errors(stream_))
        throw CudaError("tensor-parallel all-reduce: a wait for a peer's flag gave up");
    StepOut out;
    if (T > 1) {
        // merge: highest value first, lowest vocabulary index on ties (the TP = 1 order)
        std::vector<std::pair<float, uint32_t>> c;
        for (int r = 0; r < T; ++r)
            for (int k = 0; k < 2; ++k) {
                float v;
                std::memcpy(&v, &ws_.h_cand[4 * r + 2 * k + 1], 4);
                c.emplace_back(v, ws_.h_cand[4 * r + 2 * k]);
            }
        std::sort(c.begin(), c.end(), [](const auto& x, const auto& y) {
            return x.first > y.first || (x.first == y.first && x.second < y.second);
        });
        for (int i = 0; i < 2; ++i) {
            out.topk_idx[i] = c[i].second;
            out.topk_val[i] = c[i].first;
        }
    } else {
        const int n = static_cast<int>(std::min<uint32_t>(2, g.vocab));  // device top-2: winner + runner-up
        for (int i = 0; i < n; ++i) {
            out.topk_idx[i] = ws_.h_topk_idx[i];
            out.topk_val[i] = ws_.h_topk_val[i];
        }
        if (n < 2) out.topk_val[1] = -INFINITY;
    }
    out.token = out.topk_idx[0];
    out.logit = out.topk_val[0];
    out.near_tie = (out.logit - out.topk_val[1]) < 0.5f;
    return out;
}

StepOut Model::prefill(KvState& kv, const uint32_t* tokens, uint32_t count, std::vector<uint16_t>* logits_out,
                       const SampleSpec* sample) {
    constexpr uint32_t kChunk = 2048;  // model.cc:574
    const uint32_t first = std::min(kChunk, count);
    ensure_workspace(static_cast<int>(first), std::min<uint32_t>(count, 32768));
    reserve(kv, count);
    uint32_t off = 0;
    while (off < count) {
        const uint32_t take = std::min(kChunk, count - off);
        std::memcpy(ws_.h_ids, tokens + off, take * sizeof(uint32_t));
        HYB_CUDA(cudaMemcpyAsync(ws_.ids.p, ws_.h_ids, take * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
        forward_chunk(kv, static_cast<int>(take), off);
        off += take;
        if (off < count) HYB_CUDA(cudaStreamSynchronize(stream_));  // h_ids is reused
        else {
            // lm_head on the last row only: rows are independent (forward.cc:137-152)
            const bf16* last = ws_.xn.p + static_cast<size_t>(take - 1) * geo_.hidden;
            StepOut o = epilogue(last, false, nullptr, nullptr, logits_out, sample);
            kv.offset = count;
            kv.last_token = o.token;
            return o;
        }
    }
    throw std::logic_error("prefill: empty prompt");
}

int Model::verify(KvState& kv, const uint32_t* draft, int n, StepOut* outs) {
    if (n < 1 || n > kSpecMax) throw ArgError("verify: 1 to 8 draft tokens");
    if (kv.offset == 0) throw ArgError("verify requires a populated KV state (prefill first)");
    const int L = n + 1;
    if (kv.offset + L > 32768) throw std::runtime_error("decode beyond 32768 tokens is not supported");
    // the rejected tail may only overwrite ring slots no later step reads: a pass of L rows
    // needs capacity window + L - 1 (the window + kSpecMax rings hold any L <= kSpecMax + 1)
    for (const auto& c : kv.local)
        if (c.cap < geo_.window + static_cast<uint32_t>(L) - 1)
            throw std::logic_error("verify: ring capacity below window + rows - 1");
    ensure_workspace(L, kv.offset + L);
    ensure_batch_workspace(L);
    reserve(kv, static_cast<uint32_t>(L));
    ws_.h_ids[0] = kv.last_token;
    std::memcpy(ws_.h_ids + 1, draft, static_cast<size_t>(n) * sizeof(uint32_t));
    // the L rows run through the batched decode stack as consecutive positions of this
    // state; all L positions are written to the caches (a rejected tail lands in the ring
    // slack / past the committed global length and is overwritten later)
    std::vector<KvState*> rows(L, &kv);
    const std::vector<int> keys_max = stage_rows(rows.data(), L, 1);
    rows_forward(L, keys_max, &kv);
    lm_head_rows(L, outs);
    int a = 0;
    while (a < n && outs[a].token == draft[a]) ++a;
    const uint32_t committed = kv.offset + static_cast<uint32_t>(a) + 1;
    for (auto& c : kv.local) c.committed = committed;
    for (auto& c : kv.global) c.committed = committed;
    kv.offset = committed;
    kv.last_token = outs[a].token;
    return a;
}

void Model::decode_layers(KvState& kv) {
    const Geometry& g = geo_;
    const int H = static_cast<int>(g.hidden);
    const int nh = heads_local_;
    cudaStream_t st = stream_;
    const uint32_t pos = kv.offset;  // position of the token being decoded
    launch_embed_packed(ws_.ids.p, 1, embed_.packed.p, H, embed_.N, embed_scale_, ws_.h_e.p, st);
    // Tensor parallel over mapped NVLink peers: the all-reduces after o_proj and down_proj
    // run inside the qmvs (the row-parallel one stores its rows to every rank, the next
    // one's residual+norm prologue sums them); otherwise a separate all-reduce.
    const bool fused_ar = tp_.active() && tp_.fused_ready();
    QmvTpFuse dn_ar;  // the previous layer's down_proj all-reduce, consumed by the next qkv
    // qkv projection of `layer` with its input norm (and the previous layer's
    // post-MLP residual/scalar) fused into its prologue
    auto qkv_params = [&](uint32_t layer) {
        const LayerW& W = layers_[layer];
        QmvParams p;
        p.packed = W.qkv.packed.p;
        p.y = ws_.qkv.p;
        p.K = H;
        p.N = W.q_rows + W.k_rows + W.v_rows;
        p.eps = g.eps;
        p.norm_w = W.in_ln.p;
        if (layer == 0) {
            p.prologue = QmvPrologue::kNorm;
            p.x = ws_.h_e.p;
        } else {
            const LayerW& P = layers_[layer - 1];
            p.prologue = QmvPrologue::kResidNorm;
            p.x = ws_.dn.p;
            p.resid = ws_.h_b.p;
            p.post_w = P.post_ff.p;
            p.scalar = P.scalar.p;
            p.h_out = ws_.h_a.p;
            if (fused_ar) {
                p.ar_mode = 2;
                p.ar = dn_ar;
            }
        }
        return p;
    };
    size_t li = 0, gi = 0;
    for (uint32_t layer = 0; layer < g.n_layers; ++layer) {
        LayerW& W = layers_[layer];
        const int qkv_rows = W.q_rows + W.k_rows + W.v_rows;
        // residual entering this layer's attention block
        const bf16* resid = layer == 0 ? ws_.h_e.p : ws_.h_a.p;
        launch_qmv(qkv_params(layer), st, true);
        // QK-norm + RoPE + cache append + attention in one cluster kernel
        DecodeFusedParams ap;
        ap.qkv = ws_.qkv.p;
        ap.v_from_k = W.v_rows == 0;
        ap.q_norm = W.q_norm.p;
        ap.k_norm = W.k_norm.p;
        ap.inv_freq = W.inv_freq;
        ap.eps = g.eps;
        ap.pos = static_cast<int>(pos);
        ap.n_heads = nh;
        ap.n_kv = W.nkv;
        ap.hd = W.hd;
        ap.rounding = attn_rounding_;
        ap.out = ws_.attn.p;
        if (W.kind == LayerKind::Sliding) {
            LocalCache& c = kv.local[li++];
            ap.k_cache = c.k;
            ap.v_cache = c.v;
            ap.cap = static_cast<int>(c.cap);
            ap.tmap_k = &c.tk;
            ap.tmap_v = &c.tv;
            ap.n_keys = static_cast<int>(std::min(g.window, pos + 1));  // forward.cc:55-57
            c.committed = pos + 1;
        } else {
            GlobalCache& c = kv.global[gi++];
            if (c.capacity < pos + 1) throw std::runtime_error("global cache not reserved");
            ap.k_cache = c.k;
            ap.v_cache = c.v;
            ap.cap = static_cast<int>(c.capacity);
            ap.tmap_k = &c.tk;
            ap.tmap_v = &c.tv;
            ap.n_keys = static_cast<int>(pos + 1);
            c.committed = pos + 1;
        }
        if (decode_attn_fused_fits(nh, W.nkv, W.hd, ap.n_keys)) {
            launch_decode_attn_fused(ap, st, true);
        } else {
            // contexts whose scores outgrow one cluster's shared memory: separate
            // norm/RoPE/append kernel, then split-K attention over global scratch
            QkvPostParams qp;
            qp.qkv = ws_.qkv.p;
            qp.L = 1;
            qp.ld = qkv_rows;
            qp.n_heads = nh;
            qp.n_kv = W.nkv;
            qp.hd = W.hd;
            qp.v_from_k = ap.v_from_k;
            qp.q_norm = W.q_norm.p;
            qp.k_norm = W.k_norm.p;
            qp.inv_freq = W.inv_freq;
            qp.pos0 = ap.pos;
            qp.eps = g.eps;
            qp.q_out = ws_.q.p;
            qp.k_cache = ap.k_cache;
            qp.v_cache = ap.v_cache;
            qp.cache_cap = ap.cap;
            launch_qkv_post(qp, st);
            DecodeAttnParams dp;
            dp.q = ws_.q.p;
            dp.k_cache = ap.k_cache;
            dp.v_cache = ap.v_cache;
            dp.out = ws_.attn.p;
            dp.n_heads = nh;
            dp.n_kv = W.nkv;
            dp.hd = W.hd;
            dp.cap = ap.cap;
            dp.last_pos = ap.pos;
            dp.n_keys = ap.n_keys;
            dp.rounding = attn_rounding_;
            dp.scratch = ws_.attn_scratch.p;
            dp.scratch_bytes = ws_.attn_scratch_bytes;
            launch_decode_attn(dp, st);
        }
        QmvParams po;
        po.packed = W.o.packed.p;
        po.x = ws_.attn.p;
        po.y = ws_.o.p;
        po.K = W.o.K;
        po.N = H;
        // gate/up with the post-attention residual + pre-MLP norm in the prologue
        // and GeGLU in the epilogue
        QmvParams pg;
        pg.packed = W.gateup.packed.p;
        pg.x = ws_.o.p;
        pg.y = ws_.act.p;
        pg.K = H;
        pg.N = W.gateup.N;
        pg.prologue = QmvPrologue::kResidNorm;
        pg.epilogue = QmvEpilogue::kGeglu;
        pg.resid = resid;
        pg.post_w = W.post_attn.p;
        pg.scalar = nullptr;
        pg.norm_w = W.pre_ff.p;
        pg.h_out = ws_.h_b.p;
        pg.eps = g.eps;
        QmvParams pd;
        pd.packed = W.down.packed.p;
        pd.x = ws_.act.p;
        pd.y = ws_.dn.p;
        pd.K = W.down.K;
        pd.N = H;
        if (fused_ar) {
            po.ar_mode = 1;
            po.ar = tp_.next_fused_ar();
            pg.ar_mode = 2;
            pg.ar = po.ar;
            pd.ar_mode = 1;
            launch_qmv(po, st, true);
            launch_qmv(pg, st, true);
            pd.ar = tp_.next_fused_ar();
            launch_qmv(pd, st, true);
            dn_ar = pd.ar;
            last_ar_ = pd.ar;
        } else {
            launch_qmv(po, st, true);
            tp_.all_reduce_small_bf16(ws_.o.p, static_cast<size_t>(H), st, true);  // row-parallel o_proj
            launch_qmv(pg, st, true);
            launch_qmv(pd, st, true);
            tp_.all_reduce_small_bf16(ws_.dn.p, static_cast<size_t>(H), st, true);  // row-parallel down_proj
        }
    }
}

StepOut Model::decode_step(KvState& kv, std::vector<uint16_t>* logits_out, const SampleSpec* sample) {
    ensure_workspace(1, std::min<uint32_t>(kv.offset + 1, 32768));
    if (kv.offset + 1 > 32768) throw std::runtime_error("decode beyond 32768 tokens is not supported");
    reserve(kv, 1);
    ws_.h_ids[0] = kv.last_token;
    HYB_CUDA(cudaMemcpyAsync(ws_.ids.p, ws_.h_ids, sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
    decode_layers(kv);
    StepOut o = epilogue(nullptr, true, ws_.dn.p, ws_.h_b.p, logits_out, sample);
    kv.offset += 1;
    kv.last_token = o.token;
    return o;
}

// Batches up to this size project through qmv_batched; larger ones through the tcgen05 GEMM.
constexpr int kBatchQmvMax = 16;

void Model::ensure_batch_workspace(int n) {
    if (n <= bws_.cap) return;
    const Geometry& g = geo_;
    int max_k = static_cast<int>(g.hidden);
    for (const auto& L : layers_) max_k = std::max({max_k, L.q_rows, L.down.K});
    bws_.x16.reset(qmv_batch_x16_words(n, max_k));
    bws_.logits.reset(static_cast<size_t>(n) * vocab_local_);
    bws_.lm_slice.reset(n > kBatchQmvMax ? static_cast<size_t>(n) * lm_slice_rows_ : 0);
    bws_.topk_scratch.reset(static_cast<size_t>(n) * softcap_topk_scratch_floats(vocab_local_));
    bws_.topk_idx.reset(static_cast<size_t>(n) * kTopkRowStride);
    bws_.topk_val.reset(static_cast<size_t>(n) * kTopkRowStride);
    bws_.cand.reset(static_cast<size_t>(4) * n * (1 + tp_size_));
    bws_.seqs.reset(sizeof(DecodeSeq) * layers_.size() * n);
    if (bws_.h_seqs) cudaFreeHost(bws_.h_seqs);
    if (bws_.h_idx) cudaFreeHost(bws_.h_idx);
    if (bws_.h_val) cudaFreeHost(bws_.h_val);
    if (bws_.h_cand) cudaFreeHost(bws_.h_cand);
    HYB_CUDA(cudaMallocHost(&bws_.h_seqs, sizeof(DecodeSeq) * layers_.size() * n));
    HYB_CUDA(cudaMallocHost(&bws_.h_idx, sizeof(uint32_t) * kTopkRowStride * n));
    HYB_CUDA(cudaMallocHost(&bws_.h_val, sizeof(float) * kTopkRowStride * n));
    HYB_CUDA(cudaMallocHost(&bws_.h_cand, sizeof(uint32_t) * 4 * n * tp_size_));
    bws_.cap = n;
}


// lm_head over this rank's vocabulary rows for the B final-normed rows in ws_.xn, then
// soft-cap and top-2 per row (forward.cc:137-189); with tensor parallelism every rank's
// (winner, runner-up) pair is all-gathered and merged. Writes outs[0..B).
void Model::lm_head_rows(int B, StepOut* outs) {
    const Geometry& g = geo_;
    const int H = static_cast<int>(g.hidden);
    cudaStream_t st = stream_;
    if (B > kBatchQmvMax) {
        // the tcgen05 GEMM over slices of the lm_head unpacked in turn into the scratch
        for (int v0 = 0; v0 < vocab_local_; v0 += lm_slice_rows_) {
            const int n = std::min(lm_slice_rows_, vocab_local_ - v0);
            const MlxView m = unpack_rows(lm_packed_, H, v0, n, st);
            launch_quantized_matmul(ws_.xn.p, m.w, m.s, m.b, bws_.lm_slice.p, B, H, n, st);
            HYB_CUDA(cudaMemcpy2DAsync(bws_.logits.p + v0, sizeof(bf16) * vocab_local_, bws_.lm_slice.p,
                                       sizeof(bf16) * n, sizeof(bf16) * n, B, cudaMemcpyDeviceToDevice, st));
        }
    } else {
        launch_qmv_batched_x16(ws_.xn.p, B, H, H, bws_.x16.p, st);
        QmvBatchParams q;
        q.x16 = bws_.x16.p;
        q.packed = lm_packed_;
        q.y = bws_.logits.p;
        q.K = H;
        q.N = vocab_local_;
        q.B = B;
        q.ldy = vocab_local_;
        q.geglu = false;
        launch_qmv_batched(q, st);
    }
    launch_softcap_topk_rows(bws_.logits.p, B, vocab_local_, vocab_local_, g.softcap, bws_.topk_scratch.p,
                             bws_.topk_scratch.n, bws_.topk_idx.p, bws_.topk_val.p, st);
    const int T = tp_size_;
    if (T > 1) {
        tp_candidates_rows_kernel<<<1, 64, 0, st>>>(bws_.topk_idx.p, bws_.topk_val.p, B, static_cast<uint32_t>(vocab0_),
                                                     bws_.cand.p);
        HYB_LAUNCH_CHECK("tp_candidates_rows_kernel");
        tp_.all_gather_bytes(bws_.cand.p, bws_.cand.p + 4 * B, static_cast<size_t>(16) * B, st);
        HYB_CUDA(cudaMemcpyAsync(bws_.h_cand, bws_.cand.p + 4 * B, static_cast<size_t>(16) * B * T,
                                 cudaMemcpyDeviceToHost, st));
    } else {
        HYB_CUDA(cudaMemcpyAsync(bws_.h_idx, bws_.topk_idx.p, sizeof(uint32_t) * kTopkRowStride * B,
                                 cudaMemcpyDeviceToHost, st));
        HYB_CUDA(cudaMemcpyAsync(bws_.h_val, bws_.topk_val.p, sizeof(float) * kTopkRowStride * B,
                                 cudaMemcpyDeviceToHost, st));
    }
    HYB_CUDA(cudaStreamSynchronize(st));
    if (T > 1 && tp_.take_wait_errors(st))
        throw CudaError("tensor-parallel all-reduce: a wait for a peer's flag gave up");
    for (int b = 0; b < B; ++b) {
        StepOut& out = outs[b];
        out = StepOut{};
        if (T > 1) {
            // highest value first, lowest vocabulary index on ties (the TP = 1 order)
            std::vector<std::pair<float, uint32_t>> c;
            for (int r = 0; r < T; ++r)
                for (int k = 0; k < 2; ++k) {
                    const uint32_t* e = bws_.h_cand + (static_cast<size_t>(r) * B + b) * 4 + 2 * k;
                    float v;
                    std::memcpy(&v, e + 1, 4);
                    c.emplace_back(v, e[0]);
                }
            std::sort(c.begin(), c.end(), [](const auto& x, const auto& y) {
                return x.first > y.first || (x.first == y.first && x.second < y.second);
            });
            for (int i = 0; i < 2; ++i) {
                out.topk_idx[i] = c[i].second;
                out.topk_val[i] = c[i].first;
            }
        } else {
            const int n = static_cast<int>(std::min<uint32_t>(2, g.vocab));
            for (int i = 0; i < n; ++i) {
                out.topk_idx[i] = bws_.h_idx[kTopkRowStride * b + i];
                out.topk_val[i] = bws_.h_val[kTopkRowStride * b + i];
            }
            if (n < 2) out.topk_val[1] = -INFINITY;
        }
        out.token = out.topk_idx[0];
        out.logit = out.topk_val[0];
        out.near_tie = (out.logit - out.topk_val[1]) < 0.5f;
    }
}

// The layer stack for B rows whose inputs are in ws_.ids: row b's attention is described by
// entry [layer][b] of the DecodeSeq arrays (host copy bws_.h_seqs, device copy bws_.seqs),
// keys_max[layer] is its longest key range. Rows are independent sequences (batched
// decode), or, with one_seq, consecutive positions of that one sequence (verify). Leaves the
// final-normed rows in ws_.xn.
void Model::rows_forward(int B, const std::vector<int>& keys_max, const KvState* one_seq) {
    const Geometry& g = geo_;
    const int H = static_cast<int>(g.hidden), I = inter_local_;
    const int nh = heads_local_;
    cudaStream_t st = stream_;
    const DecodeSeq* hs = bws_.h_seqs;
    const DecodeSeq* dseq = reinterpret_cast<const DecodeSeq*>(bws_.seqs.p);
    // one projection for the whole batch: activations to fp16 pairs, then the packed qmv
    auto proj = [&](const bf16* x, int ldx, int K, const void* packed, int N, bf16* y, int ldy, bool geglu) {
        launch_qmv_batched_x16(x, B, ldx, K, bws_.x16.p, st);
        QmvBatchParams q;
        q.x16 = bws_.x16.p;
        q.packed = packed;
        q.y = y;
        q.K = K;
        q.N = N;
        q.B = B;
        q.ldy = ldy;
        q.geglu = geglu;
        launch_qmv_batched(q, st);
    };
    // the same through the tcgen05 GEMM over the MLX layout (split-K when its tiles cannot
    // fill the GPU); GeGLU then runs on the interleaved gate/up output. Measured on the
    // 27B shape: the batched qmv wins at 8 sequences (402 vs 286 tok/s), the GEMM at 64
    // (1045 vs 628 tok/s), where the qmv's eight MMA column groups per k-step bind it.
    auto proj_tc = [&](const bf16* x, const QLin& q, bf16* y, bool geglu) {
        const int K = q.K, N = q.N;
        const MlxView m = unpack_rows(q.packed.p, K, 0, N, st);
        if (!geglu) {
            launch_quantized_matmul(x, m.w, m.s, m.b, y, B, K, N, st);
            return;
        }
        if (qmm_tc_geglu_supported(B, K, N)) {
            launch_qmm_tc(x, m.w, m.s, m.b, y, B, K, N, st, true);
            return;
        }
        launch_quantized_matmul(x, m.w, m.s, m.b, ws_.gu.p, B, K, N, st);
        dim3 grid(std::min((N / 2 + 255) / 256, 64), B);
        geglu_interleaved_kernel<<<grid, 256, 0, st>>>(ws_.gu.p, y, N / 2);
        HYB_LAUNCH_CHECK("geglu_interleaved_kernel");
    };
    const bool tc = B > kBatchQmvMax;
    bf16* h_cur = ws_.h_a.p;
    bf16* h_alt = ws_.h_b.p;
    launch_embed_packed(ws_.ids.p, B, embed_.packed.p, H, embed_.N, embed_scale_, h_cur, st);
    launch_rms_norm(h_cur, layers_[0].in_ln.p, ws_.xn.p, B, H, g.eps, st);
    for (uint32_t layer = 0; layer < g.n_layers; ++layer) {
        LayerW& W = layers_[layer];
        const int qkv_ld = W.q_rows + W.k_rows + W.v_rows;
        if (tc) proj_tc(ws_.xn.p, W.qkv, ws_.qkv.p, false);
        else proj(ws_.xn.p, H, H, W.qkv.packed.p, qkv_ld, ws_.qkv.p, qkv_ld, false);
        if (one_seq) {
            // rows of one sequence: every row's K/V goes into the caches first (one launch),
            // so that row r's attention sees rows 0..r; the attention launch then only
            // reads the caches
            const DecodeSeq& d0 = hs[static_cast<size_t>(layer) * B];
            QkvPostParams qp;
            qp.qkv = ws_.qkv.p;
            qp.L = B;
            qp.ld = qkv_ld;
            qp.n_heads = nh;
            qp.n_kv = W.nkv;
            qp.hd = W.hd;
            qp.v_from_k = W.v_rows == 0;
            qp.q_norm = W.q_norm.p;
            qp.k_norm = W.k_norm.p;
            qp.inv_freq = W.inv_freq;
            qp.pos0 = d0.pos;
            qp.eps = g.eps;
            qp.q_out = ws_.q.p;
            qp.k_cache = d0.k_cache;
            qp.v_cache = d0.v_cache;
            qp.cache_cap = d0.cap;
            launch_qkv_post(qp, st);
        }
        // QK-norm + RoPE + cache append + attention of every sequence in one launch
        DecodeFusedParams ap;
        ap.v_from_k = W.v_rows == 0;
        ap.q_norm = W.q_norm.p;
        ap.k_norm = W.k_norm.p;
        ap.inv_freq = W.inv_freq;
        ap.eps = g.eps;
        ap.n_heads = nh;
        ap.n_kv = W.nkv;
        ap.hd = W.hd;
        ap.rounding = attn_rounding_;
        ap.seqs = dseq + static_cast<size_t>(layer) * B;
        ap.n_seq = B;
        ap.kv_ready = one_seq != nullptr;
        if (decode_attn_fused_fits(nh, W.nkv, W.hd, keys_max[layer])) {
            launch_decode_attn_fused_batch(ap, keys_max[layer], st, false);
        } else {
            // contexts beyond one cluster's shared memory: per sequence, separate
            // norm/RoPE/append and split-K attention
            for (int b = 0; b < B; ++b) {
                const DecodeSeq& d = hs[static_cast<size_t>(layer) * B + b];
                if (one_seq) {  // K/V already appended; q of row b from the append launch
                    DecodeAttnParams dp;
                    dp.q = ws_.q.p + static_cast<size_t>(b) * W.q_rows;
                    dp.k_cache = d.k_cache;
                    dp.v_cache = d.v_cache;
                    dp.out = d.out;
                    dp.n_heads = nh;
                    dp.n_kv = W.nkv;
                    dp.hd = W.hd;
                    dp.cap = d.cap;
                    dp.last_pos = d.pos;
                    dp.n_keys = d.n_keys;
                    dp.rounding = attn_rounding_;
                    dp.scratch = ws_.attn_scratch.p;
                    dp.scratch_bytes = ws_.attn_scratch_bytes;
                    launch_decode_attn(dp, st);
                    continue;
                }
                QkvPostParams qp;
                qp.qkv = d.qkv;
                qp.L = 1;
                qp.ld = qkv_ld;
                qp.n_heads = nh;
                qp.n_kv = W.nkv;
                qp.hd = W.hd;
                qp.v_from_k = ap.v_from_k;
                qp.q_norm = W.q_norm.p;
                qp.k_norm = W.k_norm.p;
                qp.inv_freq = W.inv_freq;
                qp.pos0 = d.pos;
                qp.eps = g.eps;
                qp.q_out = ws_.q.p;
                qp.k_cache = d.k_cache;
                qp.v_cache = d.v_cache;
                qp.cache_cap = d.cap;
                launch_qkv_post(qp, st);
                DecodeAttnParams dp;
                dp.q = ws_.q.p;
                dp.k_cache = d.k_cache;
                dp.v_cache = d.v_cache;
                dp.out = d.out;
                dp.n_heads = nh;
                dp.n_kv = W.nkv;
                dp.hd = W.hd;
                dp.cap = d.cap;
                dp.last_pos = d.pos;
                dp.n_keys = d.n_keys;
                dp.rounding = attn_rounding_;
                dp.scratch = ws_.attn_scratch.p;
                dp.scratch_bytes = ws_.attn_scratch_bytes;
                launch_decode_attn(dp, st);
            }
        }
        if (tc) proj_tc(ws_.attn.p, W.o, ws_.o.p, false);
        else proj(ws_.attn.p, W.q_rows, W.o.K, W.o.packed.p, H, ws_.o.p, H, false);
        tp_.all_reduce_sum_bf16(ws_.o.p, static_cast<size_t>(B) * H, st);  // row-parallel o_proj
        launch_resid_norm(ws_.o.p, W.post_attn.p, h_cur, nullptr, h_alt, W.pre_ff.p, ws_.xn.p, B, H, g.eps, st);
        if (tc) {
            proj_tc(ws_.xn.p, W.gateup, ws_.act.p, true);
            proj_tc(ws_.act.p, W.down, ws_.dn.p, false);
        } else {
            proj(ws_.xn.p, H, H, W.gateup.packed.p, W.gateup.N, ws_.act.p, I, true);
            proj(ws_.act.p, I, W.down.K, W.down.packed.p, H, ws_.dn.p, H, false);
        }
        tp_.all_reduce_sum_bf16(ws_.dn.p, static_cast<size_t>(B) * H, st);  // row-parallel down_proj
        const bf16* next_w = (layer + 1 < g.n_layers) ? layers_[layer + 1].in_ln.p : final_norm_.p;
        launch_resid_norm(ws_.dn.p, W.post_ff.p, h_alt, W.scalar.p, h_cur, next_w, ws_.xn.p, B, H, g.eps, st);
    }
}

// Attention descriptors of B rows for every layer, staged to the device with the rows'
// input tokens (ws_.h_ids): row b is state kvs[b] at position kvs[b]->offset + b * pos_step
// (pos_step 0: one step of B sequences; 1: consecutive rows of one sequence). Returns each
// layer's longest key range.
std::vector<int> Model::stage_rows(KvState* const* kvs, int B, uint32_t pos_step) {
    const Geometry& g = geo_;
    cudaStream_t st = stream_;
    DecodeSeq* hs = bws_.h_seqs;
    std::vector<int> keys_max(g.n_layers, 0);
    {
        std::vector<size_t> li(B, 0), gi(B, 0);
        for (uint32_t layer = 0; layer < g.n_layers; ++layer) {
            const LayerW& W = layers_[layer];
            const int qkv_ld = W.q_rows + W.k_rows + W.v_rows;
            for (int b = 0; b < B; ++b) {
                KvState& kv = *kvs[b];
                DecodeSeq& d = hs[static_cast<size_t>(layer) * B + b];
                const uint32_t pos = kv.offset + static_cast<uint32_t>(b) * pos_step;
                d.qkv = ws_.qkv.p + static_cast<size_t>(b) * qkv_ld;
                d.out = ws_.attn.p + static_cast<size_t>(b) * W.q_rows;
                d.pos = static_cast<int>(pos);
                if (W.kind == LayerKind::Sliding) {
                    LocalCache& c = kv.local[li[b]++];
                    d.tk = c.tk;
                    d.tv = c.tv;
                    d.k_cache = c.k;
                    d.v_cache = c.v;
                    d.cap = static_cast<int>(c.cap);
                    d.n_keys = static_cast<int>(std::min(g.window, pos + 1));  // forward.cc:55-57
                } else {
                    GlobalCache& c = kv.global[gi[b]++];
                    if (c.capacity < pos + 1) throw std::runtime_error("global cache not reserved");
                    d.tk = c.tk;
                    d.tv = c.tv;
                    d.k_cache = c.k;
                    d.v_cache = c.v;
                    d.cap = static_cast<int>(c.capacity);
                    d.n_keys = static_cast<int>(pos + 1);
                }
                keys_max[layer] = std::max(keys_max[layer], d.n_keys);
            }
        }
    }
    HYB_CUDA(cudaMemcpyAsync(bws_.seqs.p, hs, sizeof(DecodeSeq) * g.n_layers * B, cudaMemcpyHostToDevice, st));
    HYB_CUDA(cudaMemcpyAsync(ws_.ids.p, ws_.h_ids, sizeof(uint32_t) * B, cudaMemcpyHostToDevice, st));
    return keys_max;
}

void Model::decode_batch(KvState* const* kvs, int B, StepOut* outs) {
    if (B < 1 || B > kMaxDecodeBatch) throw ArgError("decode batch: 1 to 64 sequences");
    const Geometry& g = geo_;
    uint32_t max_pos = 0;
    for (int b = 0; b < B; ++b) {
        for (int c = 0; c < b; ++c)
            if (kvs[c] == kvs[b]) throw ArgError("decode batch: a state appears twice");
        if (kvs[b]->offset + 1 > 32768) throw std::runtime_error("decode beyond 32768 tokens is not supported");
        max_pos = std::max(max_pos, kvs[b]->offset);
    }
    ensure_workspace(B, std::min<uint32_t>(max_pos + 1, 32768));
    ensure_batch_workspace(B);
    for (int b = 0; b < B; ++b) {
        reserve(*kvs[b], 1);
        ws_.h_ids[b] = kvs[b]->last_token;
    }
    const std::vector<int> keys_max = stage_rows(kvs, B, 0);
    rows_forward(B, keys_max, nullptr);
    lm_head_rows(B, outs);
    for (int b = 0; b < B; ++b) {
        const StepOut& out = outs[b];
        KvState& kv = *kvs[b];
        size_t li = 0, gi = 0;
        for (uint32_t layer = 0; layer < g.n_layers; ++layer) {
            if (layers_[layer].kind == LayerKind::Sliding) kv.local[li++].committed = kv.offset + 1;
            else kv.global[gi++].committed = kv.offset + 1;
        }
        kv.offset += 1;
        kv.last_token = out.token;
    }
}

}  // namespace hyb
