// SSIM (11-tap separable Gaussian window, sigma 1.5, zero padding; C1 = 1e-4,
// C2 = 9e-4) and the fused training loss 0.8 L1 + 0.2 (1 - SSIM).
//
// Two families:
//  * the reference's five kernels with its layouts (ssim.metal:23-188), behind
//    the drop-in _SSIMFused autograd function;
//  * mg_l1_ssim_loss, the training path: two tiled kernels that never
//    materialise the 15-channel stack. Kernel 1 stages x, y with a 5-pixel
//    halo in shared memory, blurs the five moments separably, and evaluates
//    the SSIM tail and its adjoint per pixel (ssim.py:54-100), writing only
//    the three adjoint maps per channel that the chain rule needs plus the
//    loss partial sums. Kernel 2 blurs those maps back (the window is
//    symmetric, so the blur is its own adjoint) and applies the chain rule
//    dx = blur(d_mx) + 2 x blur(d_exx) + y blur(d_exy) plus the L1 sign term.
#include "kernels.cuh"

namespace mg {

namespace {

constexpr float kC1 = 0.01f * 0.01f;
constexpr float kC2 = 0.03f * 0.03f;
constexpr int kR = 5;  // window radius

// ------------------------------------------------ reference-layout kernels

__global__ void ssim_tail_forward_kernel(const float* __restrict__ b, float* __restrict__ out,
                                         int64_t npix) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= 3 * npix) return;
    const int64_t c = gid / npix, i = gid - c * npix;
    const float MX = b[(0 + c) * npix + i], MY = b[(3 + c) * npix + i];
    const float EXX = b[(6 + c) * npix + i], EYY = b[(9 + c) * npix + i];
    const float EXY = b[(12 + c) * npix + i];
    const float sxx = EXX - MX * MX, syy = EYY - MY * MY, sxy = EXY - MX * MY;
    const float A = 2.0f * MX * MY + kC1, B = 2.0f * sxy + kC2;
    const float C = MX * MX + MY * MY + kC1, D = sxx + syy + kC2;
    out[c * npix + i] = (A * B) / (C * D);
}

__global__ void ssim_tail_backward_kernel(const float* __restrict__ b,
                                          const float* __restrict__ gout,
                                          float* __restrict__ gb, int64_t npix) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= 3 * npix) return;
    const int64_t c = gid / npix, i = gid - c * npix;
    const float MX = b[(0 + c) * npix + i], MY = b[(3 + c) * npix + i];
    const float EXX = b[(6 + c) * npix + i], EYY = b[(9 + c) * npix + i];
    const float EXY = b[(12 + c) * npix + i];
    const float sxx = EXX - MX * MX, syy = EYY - MY * MY, sxy = EXY - MX * MY;
    const float A = 2.0f * MX * MY + kC1, B = 2.0f * sxy + kC2;
    const float C = MX * MX + MY * MY + kC1, D = sxx + syy + kC2;
    const float invCD = 1.0f / (C * D);
    const float S = A * B * invCD;
    const float g = gout[c * npix + i];
    const float dA = B * invCD, dB = A * invCD, dC = -S / C, dD = -S / D;
    gb[(6 + c) * npix + i] = g * dD;
    gb[(9 + c) * npix + i] = g * dD;
    gb[(12 + c) * npix + i] = g * (2.0f * dB);
    gb[(0 + c) * npix + i] = g * (2.0f * MY * (dA - dB) + 2.0f * MX * (dC - dD));
    gb[(3 + c) * npix + i] = g * (2.0f * MX * (dA - dB) + 2.0f * MY * (dC - dD));
}

__global__ void ssim_stack_blur_h_kernel(const float* __restrict__ x, const float* __restrict__ y,
                                         const float* __restrict__ w, int W, int H,
                                         float* __restrict__ out) {
    const int px = blockIdx.x * blockDim.x + threadIdx.x, py = blockIdx.y * blockDim.y + threadIdx.y;
    const int c = blockIdx.z;
    if (px >= W || py >= H) return;
    const int64_t N = (int64_t)W * H, row = (int64_t)py * W;
    float sx = 0, sy = 0, sxx = 0, syy = 0, sxy = 0;
    for (int k = -kR; k <= kR; ++k) {
        const int u = px + k;
        if (u < 0 || u >= W) continue;
        const float wk = w[k + kR];
        const float xv = x[(row + u) * 3 + c], yv = y[(row + u) * 3 + c];
        sx += wk * xv; sy += wk * yv;
        sxx += wk * xv * xv; syy += wk * yv * yv; sxy += wk * xv * yv;
    }
    const int64_t o = row + px;
    out[(0 + c) * N + o] = sx; out[(3 + c) * N + o] = sy;
    out[(6 + c) * N + o] = sxx; out[(9 + c) * N + o] = syy; out[(12 + c) * N + o] = sxy;
}

__global__ void ssim_blur15_kernel(const float* __restrict__ src, const float* __restrict__ w,
                                   int dir, int W, int H, float* __restrict__ dst) {
    const int px = blockIdx.x * blockDim.x + threadIdx.x, py = blockIdx.y * blockDim.y + threadIdx.y;
    const int ch = blockIdx.z;
    if (px >= W || py >= H) return;
    const int64_t N = (int64_t)W * H, base = ch * N;
    float s = 0;
    for (int k = -kR; k <= kR; ++k) {
        int u = px, v = py;
        if (dir == 0) u += k; else v += k;
        if (u < 0 || u >= W || v < 0 || v >= H) continue;
        s += w[k + kR] * src[base + (int64_t)v * W + u];
    }
    dst[base + (int64_t)py * W + px] = s;
}

__global__ void ssim_chain_backward_kernel(const float* __restrict__ x, const float* __restrict__ y,
                                           const float* __restrict__ d_stack, int W, int H,
                                           float* __restrict__ d_x) {
    const int px = blockIdx.x * blockDim.x + threadIdx.x, py = blockIdx.y * blockDim.y + threadIdx.y;
    const int c = blockIdx.z;
    if (px >= W || py >= H) return;
    const int64_t N = (int64_t)W * H, o = (int64_t)py * W + px;
    const float xv = x[o * 3 + c], yv = y[o * 3 + c];
    d_x[o * 3 + c] = d_stack[(0 + c) * N + o] + 2.0f * xv * d_stack[(6 + c) * N + o] +
                     yv * d_stack[(12 + c) * N + o];
}

// ------------------------------------------------------- fused training loss
//
// Tiles of kLW x kLH outputs per 256-thread block (32 x 8 threads), one colour
// channel per block (blockIdx.z). The block stages its inputs with the 5-pixel
// halo, then
//  * horizontal pass: each thread produces 4 adjacent columns of one staged
//    row from 14 inputs held in registers (16-byte shared loads; products
//    such as x*x formed once per input, not once per tap);
//  * vertical pass: each thread produces kLRows adjacent rows of one column
//    from kLRows + 10 horizontally blurred rows.

constexpr int kLW = 32;              // output tile width (one warp of columns)
constexpr int kLH = 24;              // output tile height
constexpr int kLRows = kLH / 8;      // output rows per thread in the vertical pass
constexpr int kSW = kLW + 2 * kR;    // staged width (42)
constexpr int kSH = kLH + 2 * kR;    // staged height (34)
constexpr int kSP = 44;              // staged row pitch: 16-byte rows, banks staggered
constexpr int kHItems = kSH * (kLW / 4);  // horizontal work items (row, 4-column group)

// 16 staged values from column 4g of a row (only the first 14 are used).
__device__ __forceinline__ void load16(const float* row, int g, float (&v)[16]) {
    const float4* r = reinterpret_cast<const float4*>(row) + g;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float4 t = r[k];
        v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
    }
}

// Target values. Float images are read as they are; 8-bit images as x / 255
// in float32 with IEEE division (what numpy's float32 x / 255 and the CPU
// restatement give), looked up in a 256-entry table each block fills once.
struct TargetTable {
    float v[256];
    __device__ __forceinline__ void fill() {
        const int t = threadIdx.y * blockDim.x + threadIdx.x;
        for (int i = t; i < 256; i += blockDim.x * blockDim.y)
            v[i] = __fdiv_rn((float)i, 255.0f);
    }
};
__device__ __forceinline__ float pixel_value(const float* __restrict__ src, int64_t i,
                                             const TargetTable*) {
    return src[i];
}
__device__ __forceinline__ float pixel_value(const uint8_t* __restrict__ src, int64_t i,
                                             const TargetTable* tab) {
    return tab->v[src[i]];
}

// stage_channel for a float image as 4-byte asynchronous copies (zero-filled
// outside the image); the caller commits and waits.
__device__ __forceinline__ void stage_channel_async(const float* __restrict__ src, int c, int W,
                                                    int H, int ox, int oy, float (*dst)[kSP]) {
    for (int ly = threadIdx.y; ly < kSH; ly += 8) {
        const int gy = oy + ly - kR;
        for (int lx = threadIdx.x; lx < kSP; lx += 32) {
            const int gx = ox + lx - kR;
            const bool ok = lx < kSW && gx >= 0 && gx < W && gy >= 0 && gy < H;
            const int64_t i = ok ? ((int64_t)gy * W + gx) * 3 + c : 0;
            const uint32_t d = (uint32_t)__cvta_generic_to_shared(&dst[ly][lx]);
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(d), "l"(src + i),
                         "r"(ok ? 4 : 0)
                         : "memory");
        }
    }
}

// Stages channel c of `src` (H, W, 3) around the tile at (ox, oy), zero outside.
template <typename T>
__device__ __forceinline__ void stage_channel(const T* __restrict__ src, int c, int W, int H,
                                              int ox, int oy, float (*dst)[kSP],
                                              const TargetTable* tab = nullptr) {
    for (int ly = threadIdx.y; ly < kSH; ly += 8) {
        const int gy = oy + ly - kR;
        for (int lx = threadIdx.x; lx < kSP; lx += 32) {
            const int gx = ox + lx - kR;
            const bool ok = lx < kSW && gx >= 0 && gx < W && gy >= 0 && gy < H;
            dst[ly][lx] = ok ? pixel_value(src, ((int64_t)gy * W + gx) * 3 + c, tab) : 0.f;
        }
    }
}

// Kernel 1: moments -> SSIM, its adjoint maps and the loss partial sums.
#ifndef MG_LOSS_MIN_BLOCKS
#define MG_LOSS_MIN_BLOCKS 6
#endif
// Six blocks per SM keep an 800 x 800 image (850 tiles) in one wave.
template <typename TY>
__global__ void __launch_bounds__(256, MG_LOSS_MIN_BLOCKS)
loss_moments_kernel(const float* __restrict__ x, const TY* __restrict__ y,
                    const float* __restrict__ win, int W, int H, float g_ssim,
                    float* __restrict__ adj, float* __restrict__ partial) {
    __shared__ __align__(16) float s_x[kSH][kSP];
    __shared__ __align__(16) float s_y[kSH][kSP];
    __shared__ __align__(16) float s_h[5][kSH][kLW];
    __shared__ float s_red[2][8];
    __shared__ TargetTable s_tab;
    const int tx = threadIdx.x, ty = threadIdx.y, tid = ty * 32 + tx;
    const int ox = blockIdx.x * kLW, oy = blockIdx.y * kLH;
    const int64_t npix = (int64_t)W * H;
    float wk[11];
#pragma unroll
    for (int k = 0; k < 11; ++k) wk[k] = win[k];
    float sum_s = 0.f, sum_l1 = 0.f;
    if (sizeof(TY) == 1) {
        s_tab.fill();
        __syncthreads();
    }
    {
        const int c = blockIdx.z;  // one colour channel per block
        stage_channel_async(x, c, W, H, ox, oy, s_x);  // in flight while y is staged
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        stage_channel(y, c, W, H, ox, oy, s_y, &s_tab);
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        __syncthreads();
        for (int it = tid; it < kHItems; it += 256) {
            const int row = it >> 3, g = it & 7;
            float xv[16], yv[16];
            load16(s_x[row], g, xv);
            load16(s_y[row], g, yv);
            float acc[5][4];
#pragma unroll
            for (int q = 0; q < 5; ++q)
#pragma unroll
                for (int p = 0; p < 4; ++p) acc[q][p] = 0.f;
#pragma unroll
            for (int j = 0; j < 14; ++j) {
                const float a = xv[j], b = yv[j];
                const float v5[5] = {a, b, a * a, b * b, a * b};
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const int k = j - p;
                    if (k < 0 || k > 10) continue;
#pragma unroll
                    for (int q = 0; q < 5; ++q) acc[q][p] += wk[k] * v5[q];
                }
            }
#pragma unroll
            for (int q = 0; q < 5; ++q)
                reinterpret_cast<float4*>(s_h[q][row])[g] =
                    make_float4(acc[q][0], acc[q][1], acc[q][2], acc[q][3]);
        }
        __syncthreads();
        float m[5][kLRows];
#pragma unroll
        for (int q = 0; q < 5; ++q)
#pragma unroll
            for (int p = 0; p < kLRows; ++p) m[q][p] = 0.f;
#pragma unroll
        for (int j = 0; j < kLRows + 10; ++j) {
            float hv[5];
#pragma unroll
            for (int q = 0; q < 5; ++q) hv[q] = s_h[q][ty * kLRows + j][tx];
#pragma unroll
            for (int p = 0; p < kLRows; ++p) {
                const int k = j - p;
                if (k < 0 || k > 10) continue;
#pragma unroll
                for (int q = 0; q < 5; ++q) m[q][p] += wk[k] * hv[q];
            }
        }
        const int px = ox + tx;
#pragma unroll
        for (int p = 0; p < kLRows; ++p) {
            const int ly = ty * kLRows + p, py = oy + ly;
            if (px >= W || py >= H) continue;
            const float MX = m[0][p], MY = m[1][p];
            const float sxx = m[2][p] - MX * MX, syy = m[3][p] - MY * MY;
            const float sxy = m[4][p] - MX * MY;
            const float A = 2.0f * MX * MY + kC1, B = 2.0f * sxy + kC2;
            const float C = MX * MX + MY * MY + kC1, D = sxx + syy + kC2;
            const float invCD = 1.0f / (C * D);
            const float S = A * B * invCD;
            const float dA = B * invCD, dB = A * invCD, dC = -S / C, dD = -S / D;
            const int64_t o = (int64_t)py * W + px;
            adj[(3 * c + 0) * npix + o] = g_ssim * (2.0f * MY * (dA - dB) + 2.0f * MX * (dC - dD));
            adj[(3 * c + 1) * npix + o] = g_ssim * dD;
            adj[(3 * c + 2) * npix + o] = g_ssim * (2.0f * dB);
            sum_s += S;
            sum_l1 += fabsf(s_x[ly + kR][tx + kR] - s_y[ly + kR][tx + kR]);
        }
        __syncthreads();  // s_x, s_y hold the L1 term's inputs until here
    }
    for (int o = 16; o > 0; o >>= 1) {
        sum_s += __shfl_xor_sync(0xffffffffu, sum_s, o);
        sum_l1 += __shfl_xor_sync(0xffffffffu, sum_l1, o);
    }
    if (tx == 0) { s_red[0][ty] = sum_s; s_red[1][ty] = sum_l1; }
    __syncthreads();
    if (tid == 0) {
        float a = 0.f, b = 0.f;
        for (int i = 0; i < 8; ++i) { a += s_red[0][i]; b += s_red[1][i]; }
        const int64_t blk =
            ((int64_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        partial[2 * blk + 0] = a;
        partial[2 * blk + 1] = b;
    }
}

// Kernel 2: blur the adjoint maps back and apply the chain rule + L1 term.
template <typename TY>
__global__ void __launch_bounds__(256, 6)
loss_grad_kernel(const float* __restrict__ x, const TY* __restrict__ y,
                 const float* __restrict__ adj, const float* __restrict__ win, int W, int H,
                 float g_l1, float* __restrict__ grad_x) {
    __shared__ __align__(16) float s_a[3][kSH][kSP];
    __shared__ __align__(16) float s_h[3][kSH][kLW];
    __shared__ TargetTable s_tab;
    const int tx = threadIdx.x, ty = threadIdx.y, tid = ty * 32 + tx;
    const int ox = blockIdx.x * kLW, oy = blockIdx.y * kLH;
    const int64_t npix = (int64_t)W * H;
    float wk[11];
#pragma unroll
    for (int k = 0; k < 11; ++k) wk[k] = win[k];
    if (sizeof(TY) == 1) s_tab.fill();  // ordered by the barrier after the staging
    {
        const int c = blockIdx.z;  // one colour channel per block
        // the three adjoint maps with their halo, as 4-byte asynchronous
        // copies (all in flight before one wait; zero-filled outside the
        // image)
        for (int ly = ty; ly < kSH; ly += 8) {
            const int gy = oy + ly - kR;
            for (int lx = tx; lx < kSP; lx += 32) {
                const int gx = ox + lx - kR;
                const bool ok = lx < kSW && gx >= 0 && gx < W && gy >= 0 && gy < H;
                const int64_t o = ok ? (int64_t)gy * W + gx : 0;
#pragma unroll
                for (int q = 0; q < 3; ++q) {
                    const uint32_t dst = (uint32_t)__cvta_generic_to_shared(&s_a[q][ly][lx]);
                    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(dst),
                                 "l"(adj + (3 * c + q) * npix + o), "r"(ok ? 4 : 0)
                                 : "memory");
                }
            }
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        __syncthreads();
        for (int it = tid; it < kHItems; it += 256) {
            const int row = it >> 3, g = it & 7;
            float acc[3][4];
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                float v[16];
                load16(s_a[q][row], g, v);
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    float a = 0.f;
#pragma unroll
                    for (int k = 0; k < 11; ++k) a += wk[k] * v[p + k];
                    acc[q][p] = a;
                }
            }
#pragma unroll
            for (int q = 0; q < 3; ++q)
                reinterpret_cast<float4*>(s_h[q][row])[g] =
                    make_float4(acc[q][0], acc[q][1], acc[q][2], acc[q][3]);
        }
        __syncthreads();
        float b[3][kLRows];
#pragma unroll
        for (int q = 0; q < 3; ++q)
#pragma unroll
            for (int p = 0; p < kLRows; ++p) b[q][p] = 0.f;
#pragma unroll
        for (int j = 0; j < kLRows + 10; ++j) {
            float hv[3];
#pragma unroll
            for (int q = 0; q < 3; ++q) hv[q] = s_h[q][ty * kLRows + j][tx];
#pragma unroll
            for (int p = 0; p < kLRows; ++p) {
                const int k = j - p;
                if (k < 0 || k > 10) continue;
#pragma unroll
                for (int q = 0; q < 3; ++q) b[q][p] += wk[k] * hv[q];
            }
        }
        const int px = ox + tx;
#pragma unroll
        for (int p = 0; p < kLRows; ++p) {
            const int py = oy + ty * kLRows + p;
            if (px >= W || py >= H) continue;
            const int64_t o = ((int64_t)py * W + px) * 3 + c;
            const float xv = x[o], yv = pixel_value(y, o, &s_tab);
            const float diff = xv - yv;
            const float sgn = diff > 0.f ? 1.f : (diff < 0.f ? -1.f : 0.f);
            grad_x[o] = b[0][p] + 2.0f * xv * b[1][p] + yv * b[2][p] + g_l1 * sgn;
        }
        __syncthreads();
    }
}

__global__ void loss_finish_kernel(const float* __restrict__ partial, int nblocks,
                                   float w_l1, float w_ssim, float scale, float inv_n,
                                   float* __restrict__ loss_dev) {
    __shared__ double s[2][256];
    double a = 0.0, b = 0.0;
    for (int i = threadIdx.x; i < nblocks; i += 256) {
        a += partial[2 * i];
        b += partial[2 * i + 1];
    }
    s[0][threadIdx.x] = a;
    s[1][threadIdx.x] = b;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
        if (threadIdx.x < o) {
            s[0][threadIdx.x] += s[0][threadIdx.x + o];
            s[1][threadIdx.x] += s[1][threadIdx.x + o];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const double ssim = s[0][0] * inv_n, l1 = s[1][0] * inv_n;
        // atomic: views rendered on concurrent streams add into one word
        atomicAdd(loss_dev, (float)(scale * (w_l1 * l1 + w_ssim * (1.0 - ssim))));
    }
}

dim3 grid2d(int W, int H, int t) { return dim3((W + t - 1) / t, (H + t - 1) / t, 1); }

}  // namespace

}  // namespace mg

using namespace mg;

extern "C" mg_status mg_ssim_stack_blur_h(const float* x, const float* y, const float* w,
                                          int32_t height, int32_t width, float* out,
                                          mg_stream_t stream) {
    if (width <= 0 || height <= 0) return MG_OK;
    dim3 g = grid2d(width, height, 16);
    g.z = 3;
    ssim_stack_blur_h_kernel<<<g, dim3(16, 16), 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        x, y, w, width, height, out);
    return check_launch("ssim_stack_blur_h");
}

extern "C" mg_status mg_ssim_blur15(const float* src, const float* w, int32_t dir,
                                    int32_t height, int32_t width, float* dst,
                                    mg_stream_t stream) {
    if (width <= 0 || height <= 0) return MG_OK;
    dim3 g = grid2d(width, height, 16);
    g.z = 15;
    ssim_blur15_kernel<<<g, dim3(16, 16), 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        src, w, dir, width, height, dst);
    return check_launch("ssim_blur15");
}

extern "C" mg_status mg_ssim_tail_forward(const float* b, int32_t height, int32_t width,
                                          float* out, mg_stream_t stream) {
    const int64_t npix = (int64_t)height * width;
    if (npix == 0) return MG_OK;
    ssim_tail_forward_kernel<<<ceil_div(3 * npix, 256), 256, 0,
                               reinterpret_cast<cudaStream_t>(stream)>>>(b, out, npix);
    return check_launch("ssim_tail_forward");
}

extern "C" mg_status mg_ssim_tail_backward(const float* b, const float* gout, int32_t height,
                                           int32_t width, float* gb, mg_stream_t stream) {
    const int64_t npix = (int64_t)height * width;
    if (npix == 0) return MG_OK;
    ssim_tail_backward_kernel<<<ceil_div(3 * npix, 256), 256, 0,
                                reinterpret_cast<cudaStream_t>(stream)>>>(b, gout, gb, npix);
    return check_launch("ssim_tail_backward");
}

extern "C" mg_status mg_ssim_chain_backward(const float* x, const float* y,
                                            const float* d_stack, int32_t height,
                                            int32_t width, float* d_x, mg_stream_t stream) {
    if (width <= 0 || height <= 0) return MG_OK;
    dim3 g = grid2d(width, height, 16);
    g.z = 3;
    ssim_chain_backward_kernel<<<g, dim3(16, 16), 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        x, y, d_stack, width, height, d_x);
    return check_launch("ssim_chain_backward");
}

static dim3 loss_grid(int W, int H) { return dim3((W + kLW - 1) / kLW, (H + kLH - 1) / kLH, 3); }

extern "C" size_t mg_l1_ssim_scratch_bytes(int32_t height, int32_t width) {
    const dim3 g = loss_grid(width, height);
    const size_t adj = sizeof(float) * 9 * (size_t)height * width;
    const size_t part = sizeof(float) * 2 * (size_t)g.x * g.y * g.z;
    return ((adj + 255) & ~(size_t)255) + ((part + 255) & ~(size_t)255);
}

template <typename TY>
static mg_status l1_ssim_loss_impl(const float* x, const TY* y, const float* w, int32_t height,
                                   int32_t width, float w_l1, float w_ssim, float scale,
                                   float* grad_x, float* loss_dev, void* scratch,
                                   size_t scratch_bytes, mg_stream_t stream) {
    MG_REQUIRE(height > 0 && width > 0, "l1_ssim_loss: empty image");
    MG_REQUIRE(x && y && w && grad_x && loss_dev, "l1_ssim_loss: null pointer");
    MG_REQUIRE(scratch && scratch_bytes >= mg_l1_ssim_scratch_bytes(height, width),
               "l1_ssim_loss: scratch buffer too small");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const dim3 g = loss_grid(width, height);
    const int64_t npix = (int64_t)height * width;
    float* adj = static_cast<float*>(scratch);
    float* partial = reinterpret_cast<float*>(static_cast<char*>(scratch) +
                                              ((sizeof(float) * 9 * npix + 255) & ~(size_t)255));
    const float inv_n = 1.0f / (float)(3 * npix);
    // d loss / d S_p = -scale * w_ssim / n ; d loss / d x = scale * w_l1 * sign / n
    loss_moments_kernel<TY><<<g, dim3(32, 8), 0, s>>>(x, y, w, width, height,
                                                         -scale * w_ssim * inv_n, adj, partial);
    MG_TRY(check_launch("l1_ssim_loss moments"));
    loss_grad_kernel<TY><<<g, dim3(32, 8), 0, s>>>(x, y, adj, w, width, height,
                                                      scale * w_l1 * inv_n, grad_x);
    MG_TRY(check_launch("l1_ssim_loss grad"));
    loss_finish_kernel<<<1, 256, 0, s>>>(partial, (int)(g.x * g.y * g.z), w_l1, w_ssim, scale,
                                         inv_n, loss_dev);
    return check_launch("l1_ssim_loss finish");
}

extern "C" mg_status mg_l1_ssim_loss(const float* x, const float* y, const float* w,
                                     int32_t height, int32_t width, float w_l1, float w_ssim,
                                     float scale, float* grad_x, float* loss_dev, void* scratch,
                                     size_t scratch_bytes, mg_stream_t stream) {
    return l1_ssim_loss_impl<float>(x, y, w, height, width, w_l1, w_ssim, scale, grad_x,
                                    loss_dev, scratch, scratch_bytes, stream);
}

extern "C" mg_status mg_l1_ssim_loss_u8(const float* x, const uint8_t* y, const float* w,
                                        int32_t height, int32_t width, float w_l1, float w_ssim,
                                        float scale, float* grad_x, float* loss_dev,
                                        void* scratch, size_t scratch_bytes,
                                        mg_stream_t stream) {
    return l1_ssim_loss_impl<uint8_t>(x, y, w, height, width, w_l1, w_ssim, scale, grad_x,
                                      loss_dev, scratch, scratch_bytes, stream);
}
