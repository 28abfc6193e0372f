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

constexpr int kLT = 16;               // output tile side
constexpr int kLH = kLT + 2 * kR;     // staged side with halo (26)

// Kernel 1: moments -> SSIM, its adjoint maps and the loss partial sums.
__global__ void __launch_bounds__(kLT * kLT)
loss_moments_kernel(const float* __restrict__ x, const float* __restrict__ y,
                    const float* __restrict__ win, int W, int H, float g_ssim,
                    float* __restrict__ adj, float* __restrict__ partial) {
    __shared__ float c_win[11];
    __shared__ float s_x[kLH][kLH + 1], s_y[kLH][kLH + 1];
    __shared__ float s_h[5][kLH][kLT + 1];
    __shared__ float s_red[2][kLT * kLT / 32];
    const int tx = threadIdx.x, ty = threadIdx.y, tid = ty * kLT + tx;
    const int ox = blockIdx.x * kLT, oy = blockIdx.y * kLT;
    const int px = ox + tx, py = oy + ty;
    const bool in = px < W && py < H;
    const int64_t npix = (int64_t)W * H;
    if (tid < 11) c_win[tid] = win[tid];  // published by the first barrier below
    float sum_s = 0.f, sum_l1 = 0.f;
    for (int c = 0; c < 3; ++c) {
        for (int i = tid; i < kLH * kLH; i += kLT * kLT) {
            const int ly = i / kLH, lx = i % kLH;
            const int gx = ox + lx - kR, gy = oy + ly - kR;
            const bool ok = gx >= 0 && gx < W && gy >= 0 && gy < H;
            const int64_t o = ((int64_t)gy * W + gx) * 3 + c;
            s_x[ly][lx] = ok ? x[o] : 0.f;
            s_y[ly][lx] = ok ? y[o] : 0.f;
        }
        __syncthreads();
        // horizontal pass over all kLH rows, kLT output columns
        for (int i = tid; i < kLH * kLT; i += kLT * kLT) {
            const int ly = i / kLT, lx = i % kLT;
            float a0 = 0, a1 = 0, a2 = 0, a3 = 0, a4 = 0;
#pragma unroll
            for (int k = 0; k < 11; ++k) {
                const float wk = c_win[k];
                const float xv = s_x[ly][lx + k], yv = s_y[ly][lx + k];
                a0 += wk * xv; a1 += wk * yv;
                a2 += wk * xv * xv; a3 += wk * yv * yv; a4 += wk * xv * yv;
            }
            s_h[0][ly][lx] = a0; s_h[1][ly][lx] = a1; s_h[2][ly][lx] = a2;
            s_h[3][ly][lx] = a3; s_h[4][ly][lx] = a4;
        }
        __syncthreads();
        float m[5] = {0, 0, 0, 0, 0};
#pragma unroll
        for (int k = 0; k < 11; ++k) {
            const float wk = c_win[k];
#pragma unroll
            for (int q = 0; q < 5; ++q) m[q] += wk * s_h[q][ty + k][tx];
        }
        if (in) {
            const float MX = m[0], MY = m[1];
            const float sxx = m[2] - MX * MX, syy = m[3] - MY * MY, sxy = m[4] - MX * MY;
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
            sum_l1 += fabsf(s_x[ty + kR][tx + kR] - s_y[ty + kR][tx + kR]);
        }
        __syncthreads();
    }
    // block partial sums of S and |x - y|
    for (int o = 16; o > 0; o >>= 1) {
        sum_s += __shfl_xor_sync(0xffffffffu, sum_s, o);
        sum_l1 += __shfl_xor_sync(0xffffffffu, sum_l1, o);
    }
    if ((tid & 31) == 0) { s_red[0][tid >> 5] = sum_s; s_red[1][tid >> 5] = sum_l1; }
    __syncthreads();
    if (tid == 0) {
        float a = 0.f, b = 0.f;
        for (int i = 0; i < kLT * kLT / 32; ++i) { a += s_red[0][i]; b += s_red[1][i]; }
        const int64_t blk = (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
        partial[2 * blk + 0] = a;
        partial[2 * blk + 1] = b;
    }
}

// Kernel 2: blur the adjoint maps back and apply the chain rule + L1 term.
__global__ void __launch_bounds__(kLT * kLT)
loss_grad_kernel(const float* __restrict__ x, const float* __restrict__ y,
                 const float* __restrict__ adj, const float* __restrict__ win, int W, int H,
                 float g_l1, float* __restrict__ grad_x) {
    __shared__ float c_win[11];
    __shared__ float s_a[3][kLH][kLH + 1];
    __shared__ float s_h[3][kLH][kLT + 1];
    const int tx = threadIdx.x, ty = threadIdx.y, tid = ty * kLT + tx;
    const int ox = blockIdx.x * kLT, oy = blockIdx.y * kLT;
    const int px = ox + tx, py = oy + ty;
    const bool in = px < W && py < H;
    const int64_t npix = (int64_t)W * H;
    if (tid < 11) c_win[tid] = win[tid];  // published by the first barrier below
    for (int c = 0; c < 3; ++c) {
        for (int i = tid; i < kLH * kLH; i += kLT * kLT) {
            const int ly = i / kLH, lx = i % kLH;
            const int gx = ox + lx - kR, gy = oy + ly - kR;
            const bool ok = gx >= 0 && gx < W && gy >= 0 && gy < H;
            const int64_t o = (int64_t)gy * W + gx;
#pragma unroll
            for (int q = 0; q < 3; ++q) s_a[q][ly][lx] = ok ? adj[(3 * c + q) * npix + o] : 0.f;
        }
        __syncthreads();
        for (int i = tid; i < kLH * kLT; i += kLT * kLT) {
            const int ly = i / kLT, lx = i % kLT;
            float a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
            for (int k = 0; k < 11; ++k) {
                const float wk = c_win[k];
                a0 += wk * s_a[0][ly][lx + k]; a1 += wk * s_a[1][ly][lx + k];
                a2 += wk * s_a[2][ly][lx + k];
            }
            s_h[0][ly][lx] = a0; s_h[1][ly][lx] = a1; s_h[2][ly][lx] = a2;
        }
        __syncthreads();
        float b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
        for (int k = 0; k < 11; ++k) {
            const float wk = c_win[k];
            b0 += wk * s_h[0][ty + k][tx]; b1 += wk * s_h[1][ty + k][tx];
            b2 += wk * s_h[2][ty + k][tx];
        }
        if (in) {
            const int64_t o = ((int64_t)py * W + px) * 3 + c;
            const float xv = x[o], yv = y[o];
            const float diff = xv - yv;
            const float sgn = diff > 0.f ? 1.f : (diff < 0.f ? -1.f : 0.f);
            grad_x[o] = b0 + 2.0f * xv * b1 + yv * b2 + g_l1 * sgn;
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
        *loss_dev += (float)(scale * (w_l1 * l1 + w_ssim * (1.0 - ssim)));
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

extern "C" size_t mg_l1_ssim_scratch_bytes(int32_t height, int32_t width) {
    const dim3 g = grid2d(width, height, kLT);
    const size_t adj = sizeof(float) * 9 * (size_t)height * width;
    const size_t part = sizeof(float) * 2 * (size_t)g.x * g.y;
    return ((adj + 255) & ~(size_t)255) + ((part + 255) & ~(size_t)255);
}

extern "C" mg_status mg_l1_ssim_loss(const float* x, const float* y, const float* w,
                                     int32_t height, int32_t width, float w_l1, float w_ssim,
                                     float scale, float* grad_x, float* loss_dev, void* scratch,
                                     size_t scratch_bytes, mg_stream_t stream) {
    MG_REQUIRE(height > 0 && width > 0, "l1_ssim_loss: empty image");
    MG_REQUIRE(x && y && w && grad_x && loss_dev, "l1_ssim_loss: null pointer");
    MG_REQUIRE(scratch && scratch_bytes >= mg_l1_ssim_scratch_bytes(height, width),
               "l1_ssim_loss: scratch buffer too small");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const dim3 g = grid2d(width, height, kLT);
    const int64_t npix = (int64_t)height * width;
    float* adj = static_cast<float*>(scratch);
    float* partial = reinterpret_cast<float*>(static_cast<char*>(scratch) +
                                              ((sizeof(float) * 9 * npix + 255) & ~(size_t)255));
    const float inv_n = 1.0f / (float)(3 * npix);
    // d loss / d S_p = -scale * w_ssim / n ; d loss / d x = scale * w_l1 * sign / n
    loss_moments_kernel<<<g, dim3(kLT, kLT), 0, s>>>(x, y, w, width, height,
                                                     -scale * w_ssim * inv_n, adj, partial);
    MG_TRY(check_launch("l1_ssim_loss moments"));
    loss_grad_kernel<<<g, dim3(kLT, kLT), 0, s>>>(x, y, adj, w, width, height,
                                                  scale * w_l1 * inv_n, grad_x);
    MG_TRY(check_launch("l1_ssim_loss grad"));
    loss_finish_kernel<<<1, 256, 0, s>>>(partial, (int)(g.x * g.y), w_l1, w_ssim, scale,
                                         inv_n, loss_dev);
    return check_launch("l1_ssim_loss finish");
}
