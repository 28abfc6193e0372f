// Adam updates: dense (torch.optim.Adam, adam.metal:25-42) and row-selective
// (SelectiveAdam, metal_gauss/selective_adam.py:116-186). Both are single
// HBM passes: read p, g, m, v; write p, m, v (28 B per element).
#include <cmath>

#include "kernels.cuh"

namespace mg {

namespace {

// torch's single-tensor Adam, in its operation order:
//   m.lerp_(g, 1-b1); v.mul_(b2).addcmul_(g, g, 1-b2);
//   denom = sqrt(v) / sqrt(bc2) + eps; p.addcdiv_(m, denom, -lr/bc1)
__global__ void adam_kernel(float* __restrict__ p, const float* __restrict__ g,
                            float* __restrict__ m, float* __restrict__ v, int64_t n,
                            float lr_over_bc1, float b1, float b2, float eps,
                            float sqrt_bc2) {
    const float w1 = 1.0f - b1, w2 = 1.0f - b2;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float gi = g[i];
        float mi = m[i];
        // lerp(start, end, w) with w < 0.5: start + w * (end - start)
        mi = __fadd_rn(mi, __fmul_rn(w1, __fsub_rn(gi, mi)));
        float vi = __fmul_rn(v[i], b2);
        vi = __fadd_rn(vi, __fmul_rn(__fmul_rn(w2, gi), gi));
        m[i] = mi;
        v[i] = vi;
        const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(vi), sqrt_bc2), eps);
        p[i] = __fadd_rn(p[i], __fdiv_rn(__fmul_rn(-lr_over_bc1, mi), denom));
    }
}

__global__ void selective_adam_kernel(float* __restrict__ p, const float* __restrict__ g,
                                      float* __restrict__ m, float* __restrict__ v,
                                      const float* __restrict__ steps,
                                      const uint8_t* __restrict__ visible,
                                      int64_t n_visible, int64_t rows, int64_t width,
                                      float lr, float b1, float b2, float eps, float w1,
                                      float w2) {
    const int64_t n = rows * width;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / width;
        if (r >= n_visible || visible[r] == 0) continue;
        const float k = __fadd_rn(steps[r], 1.0f);
        const float bc1 = __fsub_rn(1.0f, powf(b1, k));
        const float bc2 = __fsub_rn(1.0f, powf(b2, k));
        const float step_size = __fmul_rn(lr, __fdiv_rn(__fsqrt_rn(bc2), bc1));
        const float gi = g[i];
        const float mi = __fadd_rn(__fmul_rn(m[i], b1), __fmul_rn(gi, w1));
        const float vi = __fadd_rn(__fmul_rn(v[i], b2), __fmul_rn(__fmul_rn(gi, gi), w2));
        m[i] = mi;
        v[i] = vi;
        p[i] = __fsub_rn(p[i], __fdiv_rn(__fmul_rn(step_size, mi), __fadd_rn(__fsqrt_rn(vi), eps)));
    }
}

__global__ void advance_steps_kernel(float* __restrict__ steps,
                                     const uint8_t* __restrict__ visible, int64_t n_visible) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r < n_visible && visible[r] != 0) steps[r] = __fadd_rn(steps[r], 1.0f);
}

// SelectiveAdam's per-row bias correction sqrt(1 - b2^k) / (1 - b1^k), k the
// row's step count + 1, in the reference's operation order.
__device__ __forceinline__ float selective_row_factor(float steps, float b1, float b2) {
    const float k = __fadd_rn(steps, 1.0f);
    const float c1 = __fsub_rn(1.0f, powf(b1, k));
    const float c2 = __fsub_rn(1.0f, powf(b2, k));
    return __fdiv_rn(__fsqrt_rn(c2), c1);
}

struct AdamSegments {
    int64_t offset[MG_MAX_ADAM_SEGMENTS];
    int64_t begin[MG_MAX_ADAM_SEGMENTS];
    int64_t count[MG_MAX_ADAM_SEGMENTS];
    int32_t width[MG_MAX_ADAM_SEGMENTS];
    float lr[MG_MAX_ADAM_SEGMENTS];
};

// One launch over every segment (blockIdx.y). Selective mode (vis != null)
// follows selective_adam_kernel's arithmetic with the shared per-row step
// count; dense mode follows adam_kernel's. Each thread updates four
// consecutive elements (16-byte accesses when they are aligned); their rows
// are tracked incrementally, and a row's bias correction is computed once
// per thread however many of its elements the thread holds (sh_rest rows
// have 45), instead of once per element.
__global__ void adam_multi_kernel(float* __restrict__ p, const float* __restrict__ g,
                                  float* __restrict__ m, float* __restrict__ v, int64_t rows,
                                  AdamSegments segs, float b1, float b2, float eps, float w1,
                                  float w2, const float* __restrict__ vis,
                                  const float* __restrict__ steps,
                                  const float* __restrict__ row_factor, float bc1,
                                  float sqrt_bc2) {
    const int s = blockIdx.y;
    const int64_t off = segs.offset[s], first = segs.begin[s];
    const int width = segs.width[s];
    const float lr = segs.lr[s];
    const int64_t count = segs.count[s];
    for (int64_t k0 = 4 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x); k0 < count;
         k0 += 4 * (int64_t)gridDim.x * blockDim.x) {
        const int64_t e0 = first + k0;  // element within the segment
        const int64_t i0 = off + e0;
        const int nk = (int)min((int64_t)4, count - k0);
        const bool vec = nk == 4 && (i0 & 3) == 0;
        float gv[4], mv[4], vv[4], pv[4];
        if (vec) {
            const float4 a = *reinterpret_cast<const float4*>(g + i0);
            const float4 b = *reinterpret_cast<const float4*>(m + i0);
            const float4 c = *reinterpret_cast<const float4*>(v + i0);
            const float4 d = *reinterpret_cast<const float4*>(p + i0);
            gv[0] = a.x; gv[1] = a.y; gv[2] = a.z; gv[3] = a.w;
            mv[0] = b.x; mv[1] = b.y; mv[2] = b.z; mv[3] = b.w;
            vv[0] = c.x; vv[1] = c.y; vv[2] = c.z; vv[3] = c.w;
            pv[0] = d.x; pv[1] = d.y; pv[2] = d.z; pv[3] = d.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const bool in = j < nk;
                gv[j] = in ? g[i0 + j] : 0.f;
                mv[j] = in ? m[i0 + j] : 0.f;
                vv[j] = in ? v[i0 + j] : 0.f;
                pv[j] = in ? p[i0 + j] : 0.f;
            }
        }
        if (vis != nullptr) {
            int64_t r = e0 / width;
            int c = (int)(e0 - r * width);
            int64_t r_done = -1;
            bool live = false;
            float step_size = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j < nk) {
                    if (r != r_done) {
                        r_done = r;
                        if (row_factor) {  // precomputed once per row
                            const float f = row_factor[r];
                            live = f > 0.0f;
                            step_size = __fmul_rn(lr, f);
                        } else {
                            live = vis[r] > 0.0f;
                            if (live)
                                step_size = __fmul_rn(lr, selective_row_factor(steps[r], b1, b2));
                        }
                    }
                    if (live) {
                        const float gi = gv[j];
                        const float mi = __fadd_rn(__fmul_rn(mv[j], b1), __fmul_rn(gi, w1));
                        const float vi =
                            __fadd_rn(__fmul_rn(vv[j], b2), __fmul_rn(__fmul_rn(gi, gi), w2));
                        mv[j] = mi;
                        vv[j] = vi;
                        pv[j] = __fsub_rn(pv[j], __fdiv_rn(__fmul_rn(step_size, mi),
                                                           __fadd_rn(__fsqrt_rn(vi), eps)));
                    }
                    if (++c == width) { c = 0; ++r; }
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float gi = gv[j];
                float mi = mv[j];
                mi = __fadd_rn(mi, __fmul_rn(1.0f - b1, __fsub_rn(gi, mi)));
                const float vi =
                    __fadd_rn(__fmul_rn(vv[j], b2), __fmul_rn(__fmul_rn(1.0f - b2, gi), gi));
                mv[j] = mi;
                vv[j] = vi;
                const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(vi), sqrt_bc2), eps);
                pv[j] = __fadd_rn(pv[j], __fdiv_rn(__fmul_rn(-(lr / bc1), mi), denom));
            }
        }
        if (vec) {
            *reinterpret_cast<float4*>(m + i0) = make_float4(mv[0], mv[1], mv[2], mv[3]);
            *reinterpret_cast<float4*>(v + i0) = make_float4(vv[0], vv[1], vv[2], vv[3]);
            *reinterpret_cast<float4*>(p + i0) = make_float4(pv[0], pv[1], pv[2], pv[3]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j < nk) {
                    m[i0 + j] = mv[j];
                    v[i0 + j] = vv[j];
                    p[i0 + j] = pv[j];
                }
            }
        }
    }
}

// sqrt(1 - b2^k) / (1 - b1^k) of every visible row (0 for the others), k its
// step count + 1: the bias-correction factor of selective_adam_kernel, so
// adam_multi_kernel's threads read it instead of each forming it again.
__global__ void row_factor_kernel(const float* __restrict__ vis, const float* __restrict__ steps,
                                  int64_t rows, float b1, float b2, float* __restrict__ out) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    out[r] = vis[r] > 0.0f ? selective_row_factor(steps[r], b1, b2) : 0.0f;
}

__global__ void advance_steps_count_kernel(float* __restrict__ steps,
                                           const float* __restrict__ vis, int64_t rows) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r < rows && vis[r] > 0.0f) steps[r] = __fadd_rn(steps[r], 1.0f);
}

int grid_for(int64_t n) {
    return (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
}

}  // namespace

}  // namespace mg

using namespace mg;

extern "C" mg_status mg_adam_step(float* p, const float* g, float* m, float* v, int64_t n,
                                  float lr, float b1, float b2, float eps, float bc1,
                                  float sqrt_bc2, mg_stream_t stream) {
    if (n == 0) return MG_OK;
    MG_REQUIRE(p && g && m && v, "adam_step: null pointer");
    MG_REQUIRE(bc1 > 0.0f && sqrt_bc2 > 0.0f, "adam_step: bias corrections must be > 0");
    adam_kernel<<<grid_for(n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        p, g, m, v, n, lr / bc1, b1, b2, eps, sqrt_bc2);
    return check_launch("adam_step");
}

extern "C" mg_status mg_selective_adam_step(float* p, const float* g, float* m, float* v,
                                            const float* steps, const uint8_t* visible,
                                            int64_t n_visible, int64_t rows,
                                            int64_t row_width, float lr, float b1, float b2,
                                            float eps, mg_stream_t stream) {
    if (rows == 0 || row_width == 0) return MG_OK;
    MG_REQUIRE(p && g && m && v && steps && visible, "selective_adam_step: null pointer");
    MG_REQUIRE(n_visible <= rows, "visibility mask has more rows than the parameter");
    // (1 - b) is formed in double and rounded once, as torch does for the
    // Python scalar in `grad * (1 - b1)`.
    const float w1 = (float)(1.0 - (double)b1), w2 = (float)(1.0 - (double)b2);
    selective_adam_kernel<<<grid_for(rows * row_width), 256, 0,
                            reinterpret_cast<cudaStream_t>(stream)>>>(
        p, g, m, v, steps, visible, n_visible, rows, row_width, lr, b1, b2, eps, w1, w2);
    return check_launch("selective_adam_step");
}

extern "C" mg_status mg_selective_adam_advance_steps(float* steps, const uint8_t* visible,
                                                     int64_t n_visible, int64_t rows,
                                                     mg_stream_t stream) {
    if (n_visible == 0) return MG_OK;
    MG_REQUIRE(n_visible <= rows, "visibility mask has more rows than the parameter");
    advance_steps_kernel<<<ceil_div(n_visible, 256), 256, 0,
                           reinterpret_cast<cudaStream_t>(stream)>>>(steps, visible,
                                                                     n_visible);
    return check_launch("selective_adam_advance_steps");
}

extern "C" mg_status mg_adam_multi(float* p, const float* g, float* m, float* v, int64_t rows,
                                   const mg_adam_segment* segments, int32_t n_segments,
                                   float b1, float b2, float eps, const float* visible_count,
                                   float* steps, int64_t step, float* row_scratch,
                                   int32_t flags, mg_stream_t stream) {
    MG_REQUIRE(n_segments >= 0 && n_segments <= MG_MAX_ADAM_SEGMENTS &&
                   (n_segments == 0 || segments != nullptr),
               "adam_multi: 0..MG_MAX_ADAM_SEGMENTS segments");
    MG_REQUIRE(p && g && m && v, "adam_multi: null pointer");
    MG_REQUIRE(visible_count == nullptr || steps != nullptr, "adam_multi: selective mode needs steps");
    MG_REQUIRE(visible_count != nullptr || step >= 1, "adam_multi: dense mode needs step >= 1");
    MG_REQUIRE((flags & ~(MG_ADAM_ROW_FACTORS_READY | MG_ADAM_KEEP_STEPS)) == 0,
               "adam_multi: unknown flags");
    MG_REQUIRE(!(flags & MG_ADAM_ROW_FACTORS_READY) || row_scratch != nullptr,
               "adam_multi: MG_ADAM_ROW_FACTORS_READY needs row_scratch");
    if (rows == 0) return MG_OK;
    AdamSegments segs;
    int64_t max_count = 1;
    for (int s = 0; s < n_segments; ++s) {
        const mg_adam_segment& g = segments[s];
        MG_REQUIRE(g.width > 0 && g.offset >= 0, "adam_multi: bad segment");
        const int64_t full = rows * (int64_t)g.width;
        const int64_t b = g.elem_end > 0 ? g.elem_begin : 0;
        const int64_t e = g.elem_end > 0 ? g.elem_end : full;
        MG_REQUIRE(0 <= b && b <= e && e <= full, "adam_multi: element range outside the segment");
        segs.offset[s] = g.offset;
        segs.begin[s] = b;
        segs.count[s] = e - b;
        segs.width[s] = g.width;
        segs.lr[s] = g.lr;
        max_count = std::max(max_count, e - b);
    }
    const double bc1 = visible_count ? 1.0 : 1.0 - std::pow((double)b1, (double)step);
    const double sq = visible_count ? 1.0 : std::sqrt(1.0 - std::pow((double)b2, (double)step));
    const float w1 = (float)(1.0 - (double)b1), w2 = (float)(1.0 - (double)b2);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int gx = (int)std::min<int64_t>((max_count + 1023) / 1024, 148 * 8);
    // the row factors are formed even with no segment here: a later call of
    // the same step (MG_ADAM_ROW_FACTORS_READY) may use them
    const float* rowf = nullptr;
    if (visible_count && row_scratch) {
        if (!(flags & MG_ADAM_ROW_FACTORS_READY)) {
            row_factor_kernel<<<ceil_div(rows, 256), 256, 0, st>>>(visible_count, steps, rows, b1,
                                                                    b2, row_scratch);
            MG_TRY(check_launch("adam_multi row factors"));
        }
        rowf = row_scratch;
    }
    if (n_segments > 0) {
        adam_multi_kernel<<<dim3(std::max(gx, 1), n_segments), 256, 0, st>>>(
            p, g, m, v, rows, segs, b1, b2, eps, w1, w2, visible_count, steps, rowf,
            (float)bc1, (float)sq);
        MG_TRY(check_launch("adam_multi"));
    }
    if (visible_count && !(flags & MG_ADAM_KEEP_STEPS)) {
        advance_steps_count_kernel<<<ceil_div(rows, 256), 256, 0, st>>>(steps, visible_count, rows);
        return check_launch("adam_multi steps");
    }
    return MG_OK;
}

// ------------------------------------------------ training-loss regularisers
//
// The MCMC regularisers of the reference's training loss (train.py:393-398):
//   loss += c_opac * mean(sigmoid(logit_opac[:n])) + c_scale * mean(exp(log_scales[:n]))
// (the caller folds the ramp aux = max(0, 1 - step / (0.9 steps)) and the
// weights into c_*). One pass over the rows adds the gradients into the
// parameter gradient rows and the value into the loss word.
namespace mg {
namespace {

__global__ void __launch_bounds__(256)
regularizer_kernel(const float* __restrict__ logit, const float* __restrict__ log_scales,
                   int64_t n, float k_opac, float k_scale, float* __restrict__ d_logit,
                   float* __restrict__ d_log_scales, double* __restrict__ sums) {
    double so = 0.0, ss = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float s = 1.0f / (1.0f + expf(-logit[i]));
        so += s;
        if (k_opac != 0.0f) d_logit[i] += k_opac * (s * (1.0f - s));
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            const float e = expf(log_scales[3 * i + j]);
            ss += e;
            if (k_scale != 0.0f) d_log_scales[3 * i + j] += k_scale * e;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        so += __shfl_xor_sync(0xffffffffu, so, o);
        ss += __shfl_xor_sync(0xffffffffu, ss, o);
    }
    __shared__ double s_o[8], s_s[8];
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { s_o[warp] = so; s_s[warp] = ss; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) { so += s_o[w]; ss += s_s[w]; }
        atomicAdd(&sums[0], so);
        atomicAdd(&sums[1], ss);
    }
}

__global__ void regularizer_finish_kernel(const double* __restrict__ sums, int64_t n,
                                          float c_opac, float c_scale, float* __restrict__ loss) {
    *loss += (float)((double)c_opac * sums[0] / (double)n +
                     (double)c_scale * sums[1] / (3.0 * (double)n));
}

}  // namespace
}  // namespace mg

extern "C" mg_status mg_regularizer_grad(const float* logit_opac, const float* log_scales,
                                         int64_t n, float c_opac, float c_scale, float* d_logit,
                                         float* d_log_scales, float* loss_dev, void* scratch,
                                         size_t scratch_bytes, mg_stream_t stream) {
    using namespace mg;
    MG_REQUIRE(n >= 0, "regularizer_grad: negative count");
    if (n == 0) return MG_OK;
    MG_REQUIRE(logit_opac && log_scales && d_logit && d_log_scales && loss_dev,
               "regularizer_grad: null pointer");
    MG_REQUIRE(scratch && scratch_bytes >= 2 * sizeof(double),
               "regularizer_grad: scratch too small");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    double* sums = static_cast<double*>(scratch);
    if (cudaMemsetAsync(sums, 0, 2 * sizeof(double), st) != cudaSuccess)
        return check_launch("regularizer_grad memset");
    const float k_opac = (float)((double)c_opac / (double)n);
    const float k_scale = (float)((double)c_scale / (3.0 * (double)n));
    regularizer_kernel<<<(int)std::min<int64_t>(ceil_div(n, 256), 148 * 8), 256, 0, st>>>(
        logit_opac, log_scales, n, k_opac, k_scale, d_logit, d_log_scales, sums);
    MG_TRY(check_launch("regularizer_grad"));
    regularizer_finish_kernel<<<1, 1, 0, st>>>(sums, n, c_opac, c_scale, loss_dev);
    return check_launch("regularizer_grad finish");
}
