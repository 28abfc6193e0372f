// 3DGS-MCMC densification on the device (metal_gauss/mcmc.py): relocation of
// dead Gaussians onto live ones, growth by cloning, and the exploration noise
// on the means, each on the parameters and optimizer rows of a Gaussian
// table given as row segments (a pointer and a row width in floats), so the
// same kernels serve a dict of tensors and the training engine's flat buffers.
//
// Sampling (the reference's torch.multinomial with replacement) is inverse-CDF
// over a double-precision prefix sum of the weights with uniforms from a
// counter-based generator (splitmix64, Steele, Lea & Flood, OOPSLA 2014, of
// seed and draw index); normals for the noise come from the Box-Muller
// transform. The streams differ from torch's, so runs are reproducible per
// seed but not draw-for-draw equal to the reference's; given the same picks
// (or noise), the arithmetic is the reference's.
#include <algorithm>
#include <cmath>
#include <vector>

#include "kernels.cuh"

namespace mg {

namespace {

constexpr int kMaxSegments = 32;
constexpr int kMaxMultiplicity = 51;  // mcmc.py:36

struct Segments {
    float* ptr[kMaxSegments];
    int width[kMaxSegments];
    int count;
};

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// Uniform double in [0, 1) from draw `i` of stream `seed` (53 random bits).
__device__ __forceinline__ double uniform01(uint64_t seed, uint64_t i) {
    return (double)(splitmix64(seed ^ splitmix64(i)) >> 11) * (1.0 / 9007199254740992.0);
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// o_new = 1 - (1 - o)^(1/n) and its logit (mcmc.py:83-86), and the scale
// shrink factor of an n-way split (mcmc.py:43-50).
struct Split {
    float logit, log_ratio;
};
__device__ __forceinline__ Split split_of(float o, int n) {
    const float nf = (float)n;
    const float o_new = 1.0f - powf(fmaxf(1.0f - o, 1e-6f), 1.0f / nf);
    const float logit = logf(fminf(fmaxf(o_new, 1e-6f), 1.0f - 1e-6f) / fmaxf(1.0f - o_new, 1e-6f));
    const float denom = fmaxf(fmaxf(nf, 1.0f) * fmaxf(o_new, 1e-6f), 1e-6f);
    const float ratio = sqrtf(fminf(fmaxf(o_new / denom, 0.05f), 1.0f));
    return Split{logit, logf(ratio)};
}

// Per row < n: the sampling weight (0 for dead rows when `split_dead`) and the
// dead flag; counts rows that are dead / alive / have a non-finite weight.
__global__ void classify_kernel(const float* __restrict__ logit, int64_t n,
                                const float* __restrict__ weights, float dead_thresh,
                                int split_dead, float w_floor, double* __restrict__ w_out,
                                int32_t* __restrict__ dead_flag,
                                unsigned long long* __restrict__ stats) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    unsigned dead = 0u, alive = 0u, bad = 0u;
    if (i < n) {
        const float o = sigmoidf_(logit[i]);
        const bool is_dead = split_dead && o < dead_thresh;
        float w = weights ? fmaxf(weights[i], 0.0f) : o;
        if (weights && !isfinite(weights[i])) { bad = is_dead ? 0u : 1u; w = 0.0f; }
        if (is_dead) w = 0.0f;
        else if (w_floor > 0.0f) w = fmaxf(w, w_floor);
        w_out[i] = (double)w;
        dead_flag[i] = is_dead ? 1 : 0;
        dead = is_dead; alive = !is_dead;
    }
    dead = __reduce_add_sync(0xffffffffu, dead);
    alive = __reduce_add_sync(0xffffffffu, alive);
    bad = __reduce_add_sync(0xffffffffu, bad);
    if ((threadIdx.x & 31) == 0) {
        if (dead) atomicAdd(&stats[0], (unsigned long long)dead);
        if (alive) atomicAdd(&stats[1], (unsigned long long)alive);
        if (bad) atomicAdd(&stats[2], (unsigned long long)bad);
    }
}

// Rows that are alive fall back to weight = opacity (the reference's guard
// against non-finite or all-zero weights, mcmc.py:76-77 and :147-148).
__global__ void fallback_weights_kernel(const float* __restrict__ logit, int64_t n,
                                        const int32_t* __restrict__ dead_flag, float w_floor,
                                        double* __restrict__ w) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float o = sigmoidf_(logit[i]);
    w[i] = dead_flag[i] ? 0.0 : (double)(w_floor > 0.0f ? fmaxf(o, w_floor) : o);
}

// ---- inclusive scans (double weights, int flags): block sums, one block
// scanning them, then each block adds its offset.
constexpr int kScanBlock = 1024;

template <typename T>
__device__ __forceinline__ T block_incl_scan(T v, T* s_warp) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
    }
    if (lane == 31) s_warp[warp] = v;
    __syncthreads();
    if (warp == 0) {
        T w = lane < (int)(blockDim.x >> 5) ? s_warp[lane] : (T)0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const T y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        s_warp[lane] = w;
    }
    __syncthreads();
    if (warp > 0) v += s_warp[warp - 1];
    return v;
}

template <typename T>
__global__ void __launch_bounds__(kScanBlock) scan_block_kernel(T* __restrict__ x, int64_t n,
                                                                T* __restrict__ block_sums) {
    __shared__ T s_warp[32];
    const int64_t i = (int64_t)blockIdx.x * kScanBlock + threadIdx.x;
    T v = i < n ? x[i] : (T)0;
    v = block_incl_scan(v, s_warp);
    if (i < n) x[i] = v;
    if (threadIdx.x == kScanBlock - 1) block_sums[blockIdx.x] = v;
}

template <typename T>
__global__ void __launch_bounds__(kScanBlock) scan_sums_kernel(T* __restrict__ sums, int nb) {
    __shared__ T s_warp[32];
    T carry = 0;
    for (int base = 0; base < nb; base += kScanBlock) {
        const int i = base + threadIdx.x;
        T v = i < nb ? sums[i] : (T)0;
        v = block_incl_scan(v, s_warp) + carry;
        if (i < nb) sums[i] = v;
        __syncthreads();
        carry = __shfl_sync(0xffffffffu, v, 31);  // lane 31 of warp 31 holds the total
        if ((threadIdx.x >> 5) == 31 && (threadIdx.x & 31) == 31) s_warp[0] = v;
        __syncthreads();
        carry = s_warp[0];
        __syncthreads();
    }
}

template <typename T>
__global__ void scan_add_kernel(T* __restrict__ x, int64_t n, const T* __restrict__ sums) {
    const int64_t i = (int64_t)blockIdx.x * kScanBlock + threadIdx.x;
    if (i < n && blockIdx.x > 0) x[i] += sums[blockIdx.x - 1];
}

template <typename T>
mg_status inclusive_scan(T* x, int64_t n, T* sums, cudaStream_t st) {
    const int nb = ceil_div(n, kScanBlock);
    scan_block_kernel<T><<<nb, kScanBlock, 0, st>>>(x, n, sums);
    MG_TRY(check_launch("mcmc scan blocks"));
    scan_sums_kernel<T><<<1, kScanBlock, 0, st>>>(sums, nb);
    MG_TRY(check_launch("mcmc scan sums"));
    scan_add_kernel<T><<<nb, kScanBlock, 0, st>>>(x, n, sums);
    return check_launch("mcmc scan add");
}

// Dead row indices in order from the inclusive scan of the dead flags.
__global__ void compact_dead_kernel(const int32_t* __restrict__ flag,
                                    const int32_t* __restrict__ incl, int64_t n,
                                    int32_t* __restrict__ dead_idx) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && flag[i]) dead_idx[incl[i] - 1] = (int32_t)i;
}

// Draw k picks row r with probability w_r / sum w (first row whose inclusive
// prefix exceeds u * total); with `given`, the picks are taken as they are.
__global__ void sample_kernel(const double* __restrict__ cdf, int64_t n, int64_t k_draws,
                              uint64_t seed, const int32_t* __restrict__ given,
                              int32_t* __restrict__ pick, int32_t* __restrict__ count) {
    const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= k_draws) return;
    int32_t r;
    if (given) {
        r = given[k];
    } else {
        const double u = uniform01(seed, (uint64_t)k) * cdf[n - 1];
        int64_t lo = 0, hi = n - 1;
        while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if (cdf[mid] > u) hi = mid; else lo = mid + 1;
        }
        r = (int32_t)lo;
    }
    pick[k] = r;
    atomicAdd(&count[r], 1);
}

__device__ __forceinline__ void copy_row(const Segments& seg, int skip_a, int skip_b, int64_t dst,
                                         int64_t src) {
    for (int s = 0; s < seg.count; ++s) {
        if (s == skip_a || s == skip_b) continue;
        const int w = seg.width[s];
        const float* a = seg.ptr[s] + src * w;
        float* b = seg.ptr[s] + dst * w;
        for (int j = 0; j < w; ++j) b[j] = a[j];
    }
}

__device__ __forceinline__ void zero_row(const Segments& seg, int64_t row) {
    for (int s = 0; s < seg.count; ++s) {
        const int w = seg.width[s];
        float* b = seg.ptr[s] + row * w;
        for (int j = 0; j < w; ++j) b[j] = 0.0f;
    }
}

// Copy k: row dst_k <- row pick_k (every parameter but opacity and scales,
// which take the split's corrections), optimizer rows of dst_k zeroed.
// dst_k is dead_idx[k] (relocate) or first_dst + k (grow); n of a pick is
// clamp(count, 1, 51) + extra.
__global__ void copy_kernel(Segments params, int i_logit, int i_scales, Segments opt_rows,
                            const int32_t* __restrict__ pick, const int32_t* __restrict__ count,
                            int extra, const int32_t* __restrict__ dead_idx, int64_t first_dst,
                            int64_t k_draws) {
    const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= k_draws) return;
    const int64_t src = pick[k];
    const int64_t dst = dead_idx ? (int64_t)dead_idx[k] : first_dst + k;
    const int n = min(max(count[src], 1), kMaxMultiplicity) + extra;
    const float* logit = params.ptr[i_logit];
    const Split sp = split_of(sigmoidf_(logit[src]), n);
    copy_row(params, i_logit, i_scales, dst, src);
    const float* ls = params.ptr[i_scales];
    float* ld = params.ptr[i_scales];
    ld[3 * dst + 0] = ls[3 * src + 0] + sp.log_ratio;
    ld[3 * dst + 1] = ls[3 * src + 1] + sp.log_ratio;
    ld[3 * dst + 2] = ls[3 * src + 2] + sp.log_ratio;
    params.ptr[i_logit][dst] = sp.logit;
    zero_row(opt_rows, dst);
}

// Targets (rows picked at least once) share their job with their copies:
// the same split applied in place, optimizer rows zeroed.
__global__ void target_kernel(Segments params, int i_logit, int i_scales, Segments opt_rows,
                              const int32_t* __restrict__ count, int extra, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n || count[i] == 0) return;
    const int m = min(max(count[i], 1), kMaxMultiplicity) + extra;
    float* logit = params.ptr[i_logit];
    const Split sp = split_of(sigmoidf_(logit[i]), m);
    logit[i] = sp.logit;
    float* ls = params.ptr[i_scales];
    ls[3 * i + 0] += sp.log_ratio;
    ls[3 * i + 1] += sp.log_ratio;
    ls[3 * i + 2] += sp.log_ratio;
    zero_row(opt_rows, i);
}

// SGLD exploration (mcmc.py:166-192): eps ~ N(0, 1) per axis scaled by the
// Gaussian's scales, rotated into its frame by the normalised quaternion
// (v + 2w (u x v) + 2 u x (u x v)), gated by sigmoid(-100 (opacity - gate)).
__global__ void add_noise_kernel(float* __restrict__ means, const float* __restrict__ quats,
                                 const float* __restrict__ log_scales,
                                 const float* __restrict__ logit, int64_t n, float amp,
                                 float gate_at, uint64_t seed, const float* __restrict__ eps_in) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float o = sigmoidf_(logit[i]);
    const float gate = sigmoidf_(-100.0f * (o - gate_at));
    float e[3];
    if (eps_in) {
        e[0] = eps_in[3 * i]; e[1] = eps_in[3 * i + 1]; e[2] = eps_in[3 * i + 2];
    } else {
#pragma unroll
        for (int a = 0; a < 3; ++a) {  // Box-Muller on two uniforms per axis
            const double u1 = uniform01(seed, 6 * (uint64_t)i + 2 * a);
            const double u2 = uniform01(seed, 6 * (uint64_t)i + 2 * a + 1);
            e[a] = (float)(sqrt(-2.0 * log(1.0 - u1)) * cos(6.283185307179586 * u2));
        }
    }
#pragma unroll
    for (int a = 0; a < 3; ++a) e[a] *= expf(log_scales[3 * i + a]);
    const float4 q4 = reinterpret_cast<const float4*>(quats)[i];
    const float qn = fmaxf(sqrtf(q4.x * q4.x + q4.y * q4.y + q4.z * q4.z + q4.w * q4.w), 1e-12f);
    const float w = q4.x / qn, ux = q4.y / qn, uy = q4.z / qn, uz = q4.w / qn;
    const float tx = 2.0f * (uy * e[2] - uz * e[1]);
    const float ty = 2.0f * (uz * e[0] - ux * e[2]);
    const float tz = 2.0f * (ux * e[1] - uy * e[0]);
    const float wx = e[0] + w * tx + (uy * tz - uz * ty);
    const float wy = e[1] + w * ty + (uz * tx - ux * tz);
    const float wz = e[2] + w * tz + (ux * ty - uy * tx);
    const float k = gate * amp;
    means[3 * i + 0] += wx * k;
    means[3 * i + 1] += wy * k;
    means[3 * i + 2] += wz * k;
}

struct McmcScratch {
    double* w;
    double* wsums;
    int32_t* flag;
    int32_t* incl;
    int32_t* isums;
    int32_t* dead_idx;
    int32_t* pick;
    int32_t* count;
    unsigned long long* stats;
    size_t bytes;
};

inline size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

McmcScratch carve_mcmc(void* base, int64_t n) {
    McmcScratch s;
    char* p = static_cast<char*>(base);
    const size_t n1 = (size_t)std::max<int64_t>(n, 1);
    const size_t nb = (size_t)ceil_div((int64_t)n1, kScanBlock);
    s.stats = reinterpret_cast<unsigned long long*>(p); p += 256;
    s.w = reinterpret_cast<double*>(p); p += a256(8 * n1);
    s.wsums = reinterpret_cast<double*>(p); p += a256(8 * nb);
    s.flag = reinterpret_cast<int32_t*>(p); p += a256(4 * n1);
    s.incl = reinterpret_cast<int32_t*>(p); p += a256(4 * n1);
    s.isums = reinterpret_cast<int32_t*>(p); p += a256(4 * nb);
    s.dead_idx = reinterpret_cast<int32_t*>(p); p += a256(4 * n1);
    s.pick = reinterpret_cast<int32_t*>(p); p += a256(4 * n1);
    s.count = reinterpret_cast<int32_t*>(p); p += a256(4 * n1);
    s.bytes = (size_t)(p - static_cast<char*>(base));
    return s;
}

mg_status make_segments(const mg_row_segment* in, int32_t n, Segments& out, const char* what) {
    if (n < 0 || n > kMaxSegments)
        return fail(MG_ERR_INVALID_ARGUMENT, std::string(what) + ": 0..32 row segments");
    out.count = n;
    for (int i = 0; i < n; ++i) {
        if (in[i].ptr == nullptr || in[i].width <= 0)
            return fail(MG_ERR_INVALID_ARGUMENT, std::string(what) + ": empty row segment");
        out.ptr[i] = in[i].ptr;
        out.width[i] = in[i].width;
    }
    return MG_OK;
}

// Weights, their prefix sum and (relocate) the dead rows; returns the counts
// of dead and alive rows read back on the host.
mg_status prepare_sampling(const Segments& P, int i_logit, int64_t n, const float* weights,
                           float dead_thresh, bool split_dead, float w_floor,
                           const McmcScratch& s, cudaStream_t st, int64_t& n_dead,
                           int64_t& n_alive) {
    if (cudaMemsetAsync(s.stats, 0, 256, st) != cudaSuccess) return check_launch("mcmc stats");
    classify_kernel<<<ceil_div(n, 256), 256, 0, st>>>(P.ptr[i_logit], n, weights, dead_thresh,
                                                     split_dead ? 1 : 0, w_floor, s.w, s.flag,
                                                     s.stats);
    MG_TRY(check_launch("mcmc classify"));
    MG_TRY(inclusive_scan<double>(s.w, n, s.wsums, st));
    unsigned long long stats[3];
    double total = 0.0;
    if (cudaMemcpyAsync(stats, s.stats, sizeof(stats), cudaMemcpyDeviceToHost, st) !=
            cudaSuccess ||
        cudaMemcpyAsync(&total, s.w + (n - 1), sizeof(double), cudaMemcpyDeviceToHost, st) !=
            cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return check_launch("mcmc counts");
    n_dead = (int64_t)stats[0];
    n_alive = (int64_t)stats[1];
    if (weights && (stats[2] != 0 || !(total > 0.0))) {  // fall back to opacity
        fallback_weights_kernel<<<ceil_div(n, 256), 256, 0, st>>>(P.ptr[i_logit], n, s.flag,
                                                                 w_floor, s.w);
        MG_TRY(check_launch("mcmc fallback weights"));
        MG_TRY(inclusive_scan<double>(s.w, n, s.wsums, st));
    }
    return MG_OK;
}

}  // namespace

}  // namespace mg

using namespace mg;

extern "C" size_t mg_mcmc_scratch_bytes(int64_t n) {
    if (n < 0) return 0;
    return carve_mcmc(nullptr, n).bytes;
}

extern "C" mg_status mg_mcmc_relocate(const mg_row_segment* params, int32_t n_params,
                                      int32_t logit_index, int32_t log_scales_index,
                                      const mg_row_segment* opt_rows, int32_t n_opt_rows,
                                      int64_t n_active, float dead_thresh, const float* weights,
                                      const int32_t* picks, uint64_t seed, int64_t* moved,
                                      void* scratch, size_t scratch_bytes, mg_stream_t stream) {
    MG_REQUIRE(moved != nullptr, "mcmc_relocate: null result pointer");
    *moved = 0;
    Segments P, O;
    MG_TRY(make_segments(params, n_params, P, "mcmc_relocate"));
    MG_TRY(make_segments(opt_rows, n_opt_rows, O, "mcmc_relocate"));
    MG_REQUIRE(logit_index >= 0 && logit_index < n_params && log_scales_index >= 0 &&
                   log_scales_index < n_params && P.width[logit_index] == 1 &&
                   P.width[log_scales_index] == 3,
               "mcmc_relocate: logit (width 1) and log-scale (width 3) segments required");
    if (n_active <= 0) return MG_OK;
    MG_REQUIRE(scratch && scratch_bytes >= mg_mcmc_scratch_bytes(n_active),
               "mcmc_relocate: scratch too small");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const McmcScratch s = carve_mcmc(scratch, n_active);
    int64_t n_dead = 0, n_alive = 0;
    MG_TRY(prepare_sampling(P, logit_index, n_active, weights, dead_thresh, true, 0.0f, s, st,
                            n_dead, n_alive));
    if (n_dead == 0 || n_alive == 0) return MG_OK;
    // the dead rows in order
    if (cudaMemcpyAsync(s.incl, s.flag, 4 * (size_t)n_active, cudaMemcpyDeviceToDevice, st) !=
        cudaSuccess)
        return check_launch("mcmc flags");
    MG_TRY(inclusive_scan<int32_t>(s.incl, n_active, s.isums, st));
    compact_dead_kernel<<<ceil_div(n_active, 256), 256, 0, st>>>(s.flag, s.incl, n_active,
                                                                 s.dead_idx);
    MG_TRY(check_launch("mcmc compact"));
    if (cudaMemsetAsync(s.count, 0, 4 * (size_t)n_active, st) != cudaSuccess)
        return check_launch("mcmc counts");
    sample_kernel<<<ceil_div(n_dead, 256), 256, 0, st>>>(s.w, n_active, n_dead, seed, picks,
                                                         s.pick, s.count);
    MG_TRY(check_launch("mcmc sample"));
    copy_kernel<<<ceil_div(n_dead, 256), 256, 0, st>>>(P, logit_index, log_scales_index, O, s.pick,
                                                       s.count, 0, s.dead_idx, 0, n_dead);
    MG_TRY(check_launch("mcmc relocate copies"));
    target_kernel<<<ceil_div(n_active, 256), 256, 0, st>>>(P, logit_index, log_scales_index, O,
                                                           s.count, 0, n_active);
    MG_TRY(check_launch("mcmc relocate targets"));
    *moved = n_dead;
    return MG_OK;
}

extern "C" mg_status mg_mcmc_grow(const mg_row_segment* params, int32_t n_params,
                                  int32_t logit_index, int32_t log_scales_index,
                                  const mg_row_segment* opt_rows, int32_t n_opt_rows,
                                  int64_t n_active, int64_t target, int64_t capacity,
                                  const float* weights, const int32_t* picks, uint64_t seed,
                                  int64_t* new_active, void* scratch, size_t scratch_bytes,
                                  mg_stream_t stream) {
    MG_REQUIRE(new_active != nullptr, "mcmc_grow: null result pointer");
    *new_active = n_active;
    Segments P, O;
    MG_TRY(make_segments(params, n_params, P, "mcmc_grow"));
    MG_TRY(make_segments(opt_rows, n_opt_rows, O, "mcmc_grow"));
    MG_REQUIRE(logit_index >= 0 && logit_index < n_params && log_scales_index >= 0 &&
                   log_scales_index < n_params && P.width[logit_index] == 1 &&
                   P.width[log_scales_index] == 3,
               "mcmc_grow: logit (width 1) and log-scale (width 3) segments required");
    target = std::min(target, capacity);
    const int64_t add = target - n_active;
    if (add <= 0 || n_active <= 0) return MG_OK;
    MG_REQUIRE(scratch && scratch_bytes >= mg_mcmc_scratch_bytes(capacity),
               "mcmc_grow: scratch too small (size it for the capacity)");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const McmcScratch s = carve_mcmc(scratch, capacity);
    int64_t n_dead = 0, n_alive = 0;
    MG_TRY(prepare_sampling(P, logit_index, n_active, weights, 0.0f, false, 1e-8f, s, st, n_dead,
                            n_alive));
    if (cudaMemsetAsync(s.count, 0, 4 * (size_t)n_active, st) != cudaSuccess)
        return check_launch("mcmc counts");
    sample_kernel<<<ceil_div(add, 256), 256, 0, st>>>(s.w, n_active, add, seed, picks, s.pick,
                                                      s.count);
    MG_TRY(check_launch("mcmc sample"));
    copy_kernel<<<ceil_div(add, 256), 256, 0, st>>>(P, logit_index, log_scales_index, O, s.pick,
                                                    s.count, 1, nullptr, n_active, add);
    MG_TRY(check_launch("mcmc grow copies"));
    target_kernel<<<ceil_div(n_active, 256), 256, 0, st>>>(P, logit_index, log_scales_index, O,
                                                           s.count, 1, n_active);
    MG_TRY(check_launch("mcmc grow targets"));
    *new_active = target;
    return MG_OK;
}

extern "C" mg_status mg_mcmc_add_noise(float* means, const float* quats, const float* log_scales,
                                       const float* logit_opac, int64_t n, float lr_means,
                                       float weight, float opacity_gate, uint64_t seed,
                                       const float* eps, mg_stream_t stream) {
    MG_REQUIRE(n >= 0, "mcmc_add_noise: negative count");
    if (n == 0) return MG_OK;
    MG_REQUIRE(means && quats && log_scales && logit_opac, "mcmc_add_noise: null pointer");
    MG_REQUIRE((reinterpret_cast<uintptr_t>(quats) & 15u) == 0u,
               "mcmc_add_noise: quats must be 16-byte aligned");
    add_noise_kernel<<<ceil_div(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        means, quats, log_scales, logit_opac, n, lr_means * weight, opacity_gate, seed, eps);
    return check_launch("mcmc_add_noise");
}
