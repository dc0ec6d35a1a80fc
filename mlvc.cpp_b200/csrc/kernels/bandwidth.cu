// Bandwidth-bound kernels on channels-last FP16 tensors: elementwise unary and
// broadcast binary operators, strided copies (slice / concat / layout
// conversion), gather, pixel (un)shuffle, stand-alone ReGLU, depthwise and
// generic grouped direct convolution.
//
// Arithmetic and rounding points follow the reference operators one for one:
// unary/binary  backends/driver_cubin/kernels/elementwise.cu:1-79,
// ReGLU         backends/driver_cubin/kernels/activation.cu:1-7,
// gather        backends/driver_cubin/kernels/tensor_ops.cu:1-14,
// pixel shuffle backends/driver_cubin/kernels/tensor_ops.cu:62-116 (CRD order),
// depthwise     backends/driver_cubin/kernels/depthwise_conv.cu:1-173 (FP32
//               FMA accumulation from the bias, one FP16 rounding).
// The grids are sized as a multiple of the SM count by the host, and each
// thread walks a grid-stride loop; contiguous paths move 16 bytes per access.
#include "sm100.cuh"

namespace mlvc_b200 {

__device__ __forceinline__ float unary_op(float x, int op, float alpha, float lo, float hi)
{
    switch (op) {
    case 0: return x >= 0.0f ? x : alpha * x;
    case 1: return fminf(fmaxf(x, lo), hi);
    case 2: return 1.0f / (1.0f + expf(-x));
    case 3: return 1.0f / x;
    default: return nearbyintf(x);
    }
}

__device__ __forceinline__ float binary_op(float a, float b, int op)
{
    return op == 0 ? a + b : (op == 1 ? a * b : a - b);
}

// ------------------------------------------------------------- unary
extern "C" __global__ void mlvc_unary_f16(const __grid_constant__ ElementwiseParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const long long vecs = p.count / 8;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < vecs; i += stride) {
        uint4 v = reinterpret_cast<const uint4*>(p.a)[i];
        uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float x0, x1;
            unpack_h2(w[k], x0, x1);
            w[k] = pack_h2(unary_op(x0, p.op, p.alpha, p.lo, p.hi), unary_op(x1, p.op, p.alpha, p.lo, p.hi));
        }
        reinterpret_cast<uint4*>(p.out)[i] = v;
    }
    for (long long i = vecs * 8 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < p.count;
         i += stride)
        p.out[i] = __float2half_rn(unary_op(__half2float(p.a[i]), p.op, p.alpha, p.lo, p.hi));
}

// ------------------------------------------------------------ binary
// Same-shape operands: 16-byte vectors.
extern "C" __global__ void mlvc_binary_same_f16(const __grid_constant__ ElementwiseParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const long long vecs = p.count / 8;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < vecs; i += stride) {
        uint4 va = reinterpret_cast<const uint4*>(p.a)[i];
        const uint4 vb = reinterpret_cast<const uint4*>(p.b)[i];
        uint32_t* wa = reinterpret_cast<uint32_t*>(&va);
        const uint32_t* wb = reinterpret_cast<const uint32_t*>(&vb);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float a0, a1, b0, b1;
            unpack_h2(wa[k], a0, a1);
            unpack_h2(wb[k], b0, b1);
            wa[k] = pack_h2(binary_op(a0, b0, p.op), binary_op(a1, b1, p.op));
        }
        reinterpret_cast<uint4*>(p.out)[i] = va;
    }
    for (long long i = vecs * 8 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < p.count;
         i += stride)
        p.out[i] = __float2half_rn(binary_op(__half2float(p.a[i]), __half2float(p.b[i]), p.op));
}

// General broadcast: output is dense in (n, h, w, c) order, operands are
// addressed through per-dimension strides (0 on broadcast dimensions).  When
// the channel extent and every stride are multiples of 8, `a` is contiguous in
// c and `b` is contiguous in c or constant along it (e.g. a per-channel scale
// row, or a per-pixel value), and all three pointers are 16-byte aligned, each
// thread handles 8 channels with 16-byte accesses and 32-bit index arithmetic
// (the same per-element FP32 operation and rounding as the scalar loop).
extern "C" __global__ void mlvc_binary_bcast_f16(const __grid_constant__ ElementwiseParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const bool b_vec = p.sb[3] == 1, b_const_c = p.sb[3] == 0;
    const bool vec = p.dims[3] % 8 == 0 && p.sa[3] == 1 && (b_vec || b_const_c) && p.count < (1ll << 31) &&
                     p.sa[0] % 8 == 0 && p.sa[1] % 8 == 0 && p.sa[2] % 8 == 0 &&
                     (b_const_c || (p.sb[0] % 8 == 0 && p.sb[1] % 8 == 0 && p.sb[2] % 8 == 0)) &&
                     ((reinterpret_cast<uintptr_t>(p.a) | reinterpret_cast<uintptr_t>(p.b) |
                       reinterpret_cast<uintptr_t>(p.out)) & 15u) == 0;
    if (vec) {
        const unsigned cv = static_cast<unsigned>(p.dims[3]) / 8, W = p.dims[2], H = p.dims[1];
        const unsigned total = static_cast<unsigned>(p.count / 8);
        const unsigned stride = gridDim.x * blockDim.x;
        for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
            unsigned r = i;
            const unsigned c = (r % cv) * 8;
            r /= cv;
            const unsigned w = r % W;
            r /= W;
            const unsigned h = r % H, n = r / H;
            uint4 va = *reinterpret_cast<const uint4*>(p.a + n * p.sa[0] + h * p.sa[1] + w * p.sa[2] + c);
            const mlvc_half* bp = p.b + n * p.sb[0] + h * p.sb[1] + w * p.sb[2];
            uint32_t* wa = reinterpret_cast<uint32_t*>(&va);
            if (b_vec) {
                const uint4 vb = *reinterpret_cast<const uint4*>(bp + c);
                const uint32_t* wb = reinterpret_cast<const uint32_t*>(&vb);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    float a0, a1, b0, b1;
                    unpack_h2(wa[k], a0, a1);
                    unpack_h2(wb[k], b0, b1);
                    wa[k] = pack_h2(binary_op(a0, b0, p.op), binary_op(a1, b1, p.op));
                }
            } else {
                const float b0 = __half2float(*bp);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    float a0, a1;
                    unpack_h2(wa[k], a0, a1);
                    wa[k] = pack_h2(binary_op(a0, b0, p.op), binary_op(a1, b0, p.op));
                }
            }
            *reinterpret_cast<uint4*>(p.out + static_cast<size_t>(i) * 8) = va;
        }
        return;
    }
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < p.count; i += stride) {
        long long r = i;
        const long long c = r % p.dims[3];
        r /= p.dims[3];
        const long long w = r % p.dims[2];
        r /= p.dims[2];
        const long long h = r % p.dims[1];
        const long long n = r / p.dims[1];
        const float a = __half2float(p.a[n * p.sa[0] + h * p.sa[1] + w * p.sa[2] + c * p.sa[3]]);
        const float b = __half2float(p.b[n * p.sb[0] + h * p.sb[1] + w * p.sb[2] + c * p.sb[3]]);
        p.out[i] = __float2half_rn(binary_op(a, b, p.op));
    }
}

// -------------------------------------------------------------- copies
extern "C" __global__ void mlvc_strided_copy_f16(const __grid_constant__ CopyParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < p.count; i += stride) {
        long long r = i;
        const long long i3 = r % p.dims[3];
        r /= p.dims[3];
        const long long i2 = r % p.dims[2];
        r /= p.dims[2];
        const long long i1 = r % p.dims[1];
        const long long i0 = r / p.dims[1];
        p.dst[i0 * p.ds[0] + i1 * p.ds[1] + i2 * p.ds[2] + i3 * p.ds[3]] =
            p.src[i0 * p.ss[0] + i1 * p.ss[1] + i2 * p.ss[2] + i3 * p.ss[3]];
    }
}

// Same as above, moving 8 consecutive elements (16 bytes) per step; used when
// the innermost extent is a multiple of 8 and contiguous on both sides.  The
// index decomposition runs in 32 bits when the element count allows it (a
// 64-bit division costs several times a 32-bit one).
template <typename I>
__device__ __forceinline__ void strided_copy_v8(const CopyParams& p)
{
    const I stride = static_cast<I>(gridDim.x) * blockDim.x;
    const I inner = static_cast<I>(p.dims[3] / 8), d2 = p.dims[2], d1 = p.dims[1];
    const I total = static_cast<I>(p.count / 8);
    for (I i = static_cast<I>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        I r = i;
        const I i3 = (r % inner) * 8;
        r /= inner;
        const I i2 = r % d2;
        r /= d2;
        const I i1 = r % d1, i0 = r / d1;
        *reinterpret_cast<uint4*>(p.dst + i0 * p.ds[0] + i1 * p.ds[1] + i2 * p.ds[2] + i3) =
            *reinterpret_cast<const uint4*>(p.src + i0 * p.ss[0] + i1 * p.ss[1] + i2 * p.ss[2] + i3);
    }
}

extern "C" __global__ void mlvc_strided_copy_v8_f16(const __grid_constant__ CopyParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    if (p.count < (1ll << 31))
        strided_copy_v8<unsigned>(p);
    else
        strided_copy_v8<long long>(p);
}

// NCHW <-> NHWC with pixel (un)shuffle fused, through shared memory.  One
// block handles one device row band: 32 device pixels of one row of the NHWC
// tensor and all of its C*r*r channels, i.e. C*r rows x 32*r columns of the
// NCHW tensor.  Both global sides move 16-byte vectors in contiguous runs;
// the tile keeps host rows at a 16-byte aligned pitch.  Vector path for
// r in {1, 2}; any other r (or unaligned widths) takes the scalar path.
template <int R>
__device__ __forceinline__ void boundary_vec(const BoundaryParams& p, mlvc_half* tile)
{
    constexpr int RR = R * R;
    constexpr int kSpan = 32 * R;
    constexpr int kPitch = kSpan + 8;
    const int dh = p.h, dw = p.w, dc = p.c;
    const int hc = dc / RR, hh = dh * R, hw = dw * R;
    const int tiles_x = (dw + 31) / 32;
    const int tx = blockIdx.x % tiles_x;
    const int y = (blockIdx.x / tiles_x) % dh;
    const size_t n = blockIdx.x / (tiles_x * dh);
    const int x0 = tx * 32, nx = min(32, dw - x0);
    const int hx0 = x0 * R, hspan = nx * R;
    const int rows = hc * R;
    const int vpr = (hspan + 7) / 8;  // vectors per host row (last one may be partial)
    const int dcv = dc / 8;
    const size_t dev_base = ((n * dh + y) * static_cast<size_t>(dw) + x0) * dc;
    if (!p.to_host) {
        for (int e = threadIdx.x; e < rows * vpr; e += blockDim.x) {
            const int row = e / vpr, v = e - (e / vpr) * vpr;
            const int c = row / R, dy = row % R;
            const mlvc_half* src = p.src + ((n * hc + c) * hh + y * R + dy) * static_cast<size_t>(hw) + hx0 + v * 8;
            mlvc_half* dst = tile + row * kPitch + v * 8;
            if (v * 8 + 8 <= hspan)
                *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
            else
                for (int i = 0; v * 8 + i < hspan; ++i)
                    dst[i] = src[i];
        }
        __syncthreads();
        for (int e = threadIdx.x; e < nx * dcv; e += blockDim.x) {
            const int j = e / dcv, kv = e - (e / dcv) * dcv;
            uint4 o;
            if constexpr (R >= 2) {
                // device channels kv*8 .. kv*8+7 = 8/R runs of R sub-pixels dx
                // (c, dy fixed per run), each contiguous in one tile row
                uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
                for (int q = 0; q < 8 / R; ++q) {
                    const int k = kv * 8 + q * R;  // device channel c*R*R + dy*R
                    const int c = k / RR, dy = (k % RR) / R;
                    const mlvc_half* src = tile + (c * R + dy) * kPitch + j * R;
                    if constexpr (R == 8) {
                        o = *reinterpret_cast<const uint4*>(src);
                    } else if constexpr (R == 4) {
                        const uint2 v = *reinterpret_cast<const uint2*>(src);
                        ow[2 * q] = v.x;
                        ow[2 * q + 1] = v.y;
                    } else {
                        ow[q] = *reinterpret_cast<const uint32_t*>(src);
                    }
                }
            } else {
                uint16_t h[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)  // device channel kv*8+i = host row, column j
                    h[i] = reinterpret_cast<const uint16_t*>(tile)[(kv * 8 + i) * kPitch + j];
                o.x = h[0] | (static_cast<uint32_t>(h[1]) << 16);
                o.y = h[2] | (static_cast<uint32_t>(h[3]) << 16);
                o.z = h[4] | (static_cast<uint32_t>(h[5]) << 16);
                o.w = h[6] | (static_cast<uint32_t>(h[7]) << 16);
            }
            *reinterpret_cast<uint4*>(p.dst + dev_base + static_cast<size_t>(e) * 8) = o;
        }
    } else {
        for (int e = threadIdx.x; e < nx * dcv; e += blockDim.x) {
            const int j = e / dcv, kv = e - (e / dcv) * dcv;
            const uint4 v = *reinterpret_cast<const uint4*>(p.src + dev_base + static_cast<size_t>(e) * 8);
            const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
            if constexpr (R >= 2) {
                // 8/R runs of R sub-pixels, each contiguous in one tile row
#pragma unroll
                for (int q = 0; q < 8 / R; ++q) {
                    const int k = kv * 8 + q * R;
                    const int c = k / RR, dy = (k % RR) / R;
                    mlvc_half* dst = tile + (c * R + dy) * kPitch + j * R;
                    if constexpr (R == 8)
                        *reinterpret_cast<uint4*>(dst) = v;
                    else if constexpr (R == 4)
                        *reinterpret_cast<uint2*>(dst) = make_uint2(w4[2 * q], w4[2 * q + 1]);
                    else
                        *reinterpret_cast<uint32_t*>(dst) = w4[q];
                }
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    reinterpret_cast<uint16_t*>(tile)[(kv * 8 + i) * kPitch + j] =
                        static_cast<uint16_t>(w4[i / 2] >> (16 * (i % 2)));
            }
        }
        __syncthreads();
        for (int e = threadIdx.x; e < rows * vpr; e += blockDim.x) {
            const int row = e / vpr, v = e - (e / vpr) * vpr;
            const int c = row / R, dy = row % R;
            mlvc_half* dst = p.dst + ((n * hc + c) * hh + y * R + dy) * static_cast<size_t>(hw) + hx0 + v * 8;
            const mlvc_half* src = tile + row * kPitch + v * 8;
            if (v * 8 + 8 <= hspan)
                *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
            else
                for (int i = 0; v * 8 + i < hspan; ++i)
                    dst[i] = src[i];
        }
    }
}

__device__ __forceinline__ void boundary_scalar(const BoundaryParams& p, mlvc_half* tile)
{
    const int r = p.r, rr = r * r, span = 32 * r, pitch = span + 1;
    const int dh = p.h, dw = p.w, dc = p.c;           // device NHWC extents
    const int hc = dc / rr, hh = dh * r, hw = dw * r;  // host NCHW extents
    const int tiles_x = (dw + 31) / 32;
    const int band = blockIdx.x;
    const int tx = band % tiles_x;
    const int y = (band / tiles_x) % dh;
    const long long n = band / (tiles_x * dh);
    const int x0 = tx * 32, nx = min(32, dw - x0);
    const int hx0 = x0 * r, hspan = nx * r;
    const int host_elems = hc * r * hspan;
    const int dev_elems = nx * dc;
    if (!p.to_host) {
        for (int e = threadIdx.x; e < host_elems; e += blockDim.x) {
            const int col = e % hspan, row = e / hspan;  // row = c*r + dy
            const int c = row / r, dy = row % r;
            tile[row * pitch + col] = p.src[((n * hc + c) * hh + y * r + dy) * static_cast<long long>(hw) + hx0 + col];
        }
        __syncthreads();
        mlvc_half* dst = p.dst + ((n * dh + y) * static_cast<long long>(dw) + x0) * dc;
        for (int e = threadIdx.x; e < dev_elems; e += blockDim.x) {
            const int k = e % dc, j = e / dc;  // device pixel j, channel k = c*r*r + dy*r + dx
            const int c = k / rr, dy = (k % rr) / r, dx = k % r;
            dst[e] = tile[(c * r + dy) * pitch + j * r + dx];
        }
    } else {
        const mlvc_half* src = p.src + ((n * dh + y) * static_cast<long long>(dw) + x0) * dc;
        for (int e = threadIdx.x; e < dev_elems; e += blockDim.x) {
            const int k = e % dc, j = e / dc;
            const int c = k / rr, dy = (k % rr) / r, dx = k % r;
            tile[(c * r + dy) * pitch + j * r + dx] = src[e];
        }
        __syncthreads();
        for (int e = threadIdx.x; e < host_elems; e += blockDim.x) {
            const int col = e % hspan, row = e / hspan;
            const int c = row / r, dy = row % r;
            p.dst[((n * hc + c) * hh + y * r + dy) * static_cast<long long>(hw) + hx0 + col] = tile[row * pitch + col];
        }
    }
}

// -------------------------------------------------- recurrent feature update
// The eleven operators of the recurrent-feature update (three channel slices,
// two sigmoids, six binary operators) plus the concat of their two results,
// one thread per 8 channels of a pixel.  Every operator rounds to FP16 as the
// stand-alone kernels do (same unary_op / binary_op), so the result is
// bit-identical to running them one by one (reference fused form:
// backends/driver_cubin/kernels/recurrent_feature.cu:5-107).
extern "C" __global__ void __launch_bounds__(256) mlvc_feature_update_f16(const __grid_constant__ FeatureUpdateParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const int cv = p.c / 8;
    const long long total = p.pixels * cv;
    auto rnd = [](float v) { return __half2float(__float2half_rn(v)); };
    const float one = rnd(p.one);
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long px = i / cv;
        const int c8 = static_cast<int>(i - px * cv) * 8;
        const mlvc_half* s = p.src + px * 3 * p.c + c8;
        const uint4 av = *reinterpret_cast<const uint4*>(s);
        const uint4 bv = *reinterpret_cast<const uint4*>(s + p.c);
        const uint4 cv4 = *reinterpret_cast<const uint4*>(s + 2 * p.c);
        const uint4 hv = *reinterpret_cast<const uint4*>(p.history + px * p.c + c8);
        const uint4 sv = *reinterpret_cast<const uint4*>(p.scale + c8);
        const uint32_t* aw = reinterpret_cast<const uint32_t*>(&av);
        const uint32_t* bw = reinterpret_cast<const uint32_t*>(&bv);
        const uint32_t* cw = reinterpret_cast<const uint32_t*>(&cv4);
        const uint32_t* hw = reinterpret_cast<const uint32_t*>(&hv);
        const uint32_t* sw = reinterpret_cast<const uint32_t*>(&sv);
        uint4 scaled_v, blended_v;
        uint32_t* so = reinterpret_cast<uint32_t*>(&scaled_v);
        uint32_t* bo = reinterpret_cast<uint32_t*>(&blended_v);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float a[2], b[2], c[2], h[2], sc[2], sv2[2], bl[2];
            unpack_h2(aw[k], a[0], a[1]);
            unpack_h2(bw[k], b[0], b[1]);
            unpack_h2(cw[k], c[0], c[1]);
            unpack_h2(hw[k], h[0], h[1]);
            unpack_h2(sw[k], sv2[0], sv2[1]);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float sig_b = rnd(unary_op(b[j], 2, 0.0f, 0.0f, 0.0f));
                const float sig_c = rnd(unary_op(c[j], 2, 0.0f, 0.0f, 0.0f));
                const float weighted_b = rnd(binary_op(sig_b, h[j], 1));
                const float inverse_gate = rnd(binary_op(one, sig_b, 2));
                const float weighted_a = rnd(binary_op(inverse_gate, a[j], 1));
                bl[j] = rnd(binary_op(weighted_b, weighted_a, 0));
                const float gated = rnd(binary_op(sig_c, bl[j], 1));
                sc[j] = binary_op(gated, sv2[j], 1);
            }
            so[k] = pack_h2(sc[0], sc[1]);
            bo[k] = pack_h2(bl[0], bl[1]);
        }
        if (p.concat) {
            *reinterpret_cast<uint4*>(p.concat + px * 2 * p.c + c8) = scaled_v;
            *reinterpret_cast<uint4*>(p.concat + px * 2 * p.c + p.c + c8) = blended_v;
        }
        if (p.scaled)
            *reinterpret_cast<uint4*>(p.scaled + px * p.c + c8) = scaled_v;
        if (p.blended)
            *reinterpret_cast<uint4*>(p.blended + px * p.c + c8) = blended_v;
    }
}

// ------------------------------------------------- latent quantisation tails
// The two quantisation tails of the MLVC encoder (nineteen and fifteen graph
// operators), one thread per 8 channels q of a pixel; every operator rounds to
// FP16 through the stand-alone kernels' unary_op / binary_op, so the results
// are bit-identical to running the operators one by one.
namespace {

struct Vec8 {
    float v[8];
};

__device__ __forceinline__ Vec8 load8(const mlvc_half* p)
{
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&u);
    Vec8 r;
#pragma unroll
    for (int k = 0; k < 4; ++k)
        unpack_h2(w[k], r.v[2 * k], r.v[2 * k + 1]);
    return r;
}

__device__ __forceinline__ void store8(mlvc_half* p, const Vec8& x)
{
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k)
        w[k] = pack_h2(x.v[2 * k], x.v[2 * k + 1]);
    *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ float rnd16(float v) { return __half2float(__float2half_rn(v)); }

}  // namespace

extern "C" __global__ void __launch_bounds__(256) mlvc_y0_tail_f16(const __grid_constant__ QuantTailParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const int Q = p.q, qv = Q / 8;
    const long long total = p.pixels * qv;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long px = i / qv;
        const int q = static_cast<int>(i - px * qv) * 8;
        const mlvc_half* prior = p.prior + px * 4 * Q;
        Vec8 clip[2], norm[2], s[2], u[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const Vec8 pr = load8(prior + j * Q + q), lat = load8(p.latent + px * 2 * Q + j * Q + q);
            const Vec8 tail = load8(prior + 2 * Q + j * Q + q), qs = load8(p.qscale + px * 2 * Q + j * Q + q);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                clip[j].v[k] = rnd16(unary_op(pr.v[k], 1, 0.0f, p.clip_lo, INFINITY));
                const float rec = rnd16(unary_op(clip[j].v[k], 3, 0.0f, 0.0f, 0.0f));
                norm[j].v[k] = rnd16(binary_op(lat.v[k], rec, 1));
                s[j].v[k] = rnd16(binary_op(rnd16(binary_op(norm[j].v[k], tail.v[k], 2)), qs.v[k], 1));
            }
        }
        Vec8 y;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            y.v[k] = rnd16(unary_op(rnd16(binary_op(s[0].v[k], s[1].v[k], 0)), 4, 0.0f, 0.0f, 0.0f));
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const Vec8 tail = load8(prior + 2 * Q + j * Q + q);
            const Vec8 us = load8((j ? p.uscale1 : p.uscale0) + px * Q + q);
#pragma unroll
            for (int k = 0; k < 8; ++k)
                u[j].v[k] = binary_op(rnd16(binary_op(y.v[k], tail.v[k], 0)), us.v[k], 1);
        }
        store8(p.y_raw + px * Q + q, y);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            if (p.normalized_out)
                store8(p.normalized_out + px * 2 * Q + j * Q + q, norm[j]);
            if (p.clipped_out)
                store8(p.clipped_out + px * 2 * Q + j * Q + q, clip[j]);
            if (p.concat2_out)
                store8(p.concat2_out + px * 2 * Q + j * Q + q, u[j]);
            store8(p.concat3 + px * 6 * Q + j * Q + q, u[j]);
        }
        // concat3's prior part: channels 2Q .. 6Q
#pragma unroll
        for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(p.concat3 + px * 6 * Q + 2 * Q + j * Q + q) =
                *reinterpret_cast<const uint4*>(prior + j * Q + q);
    }
}

extern "C" __global__ void __launch_bounds__(256) mlvc_y1_tail_f16(const __grid_constant__ QuantTailParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const int Q = p.q, qv = Q / 8;
    const long long total = p.pixels * qv;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long px = i / qv;
        const int q = static_cast<int>(i - px * qv) * 8;
        const long long b2 = px * 2 * Q;
        Vec8 s[2], pr[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const Vec8 n = load8(p.normalized + b2 + j * Q + q), qs = load8(p.qscale + b2 + j * Q + q);
            pr[j] = load8(p.prior + b2 + j * Q + q);
#pragma unroll
            for (int k = 0; k < 8; ++k)
                s[j].v[k] = rnd16(binary_op(rnd16(binary_op(n.v[k], pr[j].v[k], 2)), qs.v[k], 1));
        }
        Vec8 y;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            y.v[k] = rnd16(unary_op(rnd16(binary_op(s[0].v[k], s[1].v[k], 0)), 4, 0.0f, 0.0f, 0.0f));
        store8(p.y_raw + px * Q + q, y);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const Vec8 us = load8((j ? p.uscale1 : p.uscale0) + px * Q + q);
            const Vec8 c2 = load8(p.concat2_in + b2 + j * Q + q), cl = load8(p.clipped_in + b2 + j * Q + q);
            Vec8 r;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float upd = rnd16(binary_op(rnd16(binary_op(y.v[k], pr[j].v[k], 0)), us.v[k], 1));
                r.v[k] = binary_op(rnd16(binary_op(c2.v[k], upd, 0)), cl.v[k], 1);
            }
            store8(p.result + b2 + j * Q + q, r);
        }
    }
}

// ------------------------------------------------- entropy-coder inputs
// Scale extraction (reference: extract_scales, core/src/scales.cpp:25-105).
// One thread per output element (c, y, x), c < latent / 2: the base scales of
// hyper-latent channels c / repeat ("first") and (c + latent / 2) / repeat
// ("second") at the nearest z position, clamp(trunc(|z|), 0, max_index); a
// non-finite z gives INT_MIN, the reference's compiled result for its
// undefined float -> int cast there.  scales_0 takes first where x + y is
// even, scales_1 the other one.
__device__ __forceinline__ int32_t base_scale(const ScaleParams& p, int ch, int zy, int zx)
{
    const float a = fabsf(__half2float(p.z[(static_cast<long long>(ch) * p.z_height + zy) * p.z_width + zx]));
    if (!isfinite(a))
        return -2147483647 - 1;  // INT_MIN
    return min(max(__float2int_rz(a), 0), p.max_index);
}

__device__ __forceinline__ void scale_pair(const ScaleParams& p, int c, int y, int x, int32_t& s0, int32_t& s1)
{
    const int half = p.latent / 2;
    const int zy = min(y / p.spatial, p.z_height - 1), zx = min(x / p.spatial, p.z_width - 1);
    const int32_t first = base_scale(p, c / p.repeat, zy, zx);
    const int32_t second = base_scale(p, (c + half) / p.repeat, zy, zx);
    const bool even = ((x + y) & 1) == 0;
    s0 = even ? first : second;
    s1 = even ? second : first;
}

extern "C" __global__ void __launch_bounds__(256) mlvc_extract_scales(const __grid_constant__ ScaleParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const long long total = static_cast<long long>(p.latent / 2) * p.y_height * p.y_width;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    if (p.vec4) {
        // four consecutive x of one row per thread, one 16-byte store per plane
        // (host: y_width % 4 == 0, both planes 16-byte aligned)
        const int qw = p.y_width / 4;
        for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total / 4; i += stride) {
            const int x0 = static_cast<int>(i % qw) * 4;
            const long long t = i / qw;
            const int y = static_cast<int>(t % p.y_height);
            const int c = static_cast<int>(t / p.y_height);
            int32_t a[4], b[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
                scale_pair(p, c, y, x0 + k, a[k], b[k]);
            reinterpret_cast<int4*>(p.scales_0)[i] = make_int4(a[0], a[1], a[2], a[3]);
            reinterpret_cast<int4*>(p.scales_1)[i] = make_int4(b[0], b[1], b[2], b[3]);
        }
        return;
    }
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total; i += stride) {
        const int x = static_cast<int>(i % p.y_width);
        const long long t = i / p.y_width;
        int32_t a, b;
        scale_pair(p, static_cast<int>(t / p.y_height), static_cast<int>(t % p.y_height), x, a, b);
        p.scales_0[i] = a;
        p.scales_1[i] = b;
    }
}

// FP16 latents -> int32 entropy symbols (reference: integer_values,
// core/src/entropy.cpp:201-226): truncation; a value that is not finite or
// lies outside [-32768, 32767] raises the out-of-range flag, which the host
// turns into the reference's error (that element's symbol is not written).
__device__ __forceinline__ bool symbol_of(float v, int32_t& out)
{
    if (!(v >= -32768.0f && v <= 32767.0f))  // also true for NaN
        return false;
    out = __float2int_rz(v);
    return true;
}

extern "C" __global__ void __launch_bounds__(256) mlvc_integer_values_f16(const __grid_constant__ IntegerValuesParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    bool bad = false;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
    // vector body: 8 values per thread (one 16-byte load, two 16-byte stores;
    // host: both pointers 16-byte aligned), then the scalar tail
    const long long nvec = p.vec8 ? p.count / 8 : 0;
    for (long long i = tid; i < nvec; i += stride) {
        const uint4 raw = reinterpret_cast<const uint4*>(p.src)[i];
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
        int32_t o[8];
        bool ok[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
            ok[2 * k] = symbol_of(f.x, o[2 * k]);
            ok[2 * k + 1] = symbol_of(f.y, o[2 * k + 1]);
        }
        bool all = true;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            all = all && ok[k];
        if (all) {
            reinterpret_cast<int4*>(p.dst)[2 * i] = make_int4(o[0], o[1], o[2], o[3]);
            reinterpret_cast<int4*>(p.dst)[2 * i + 1] = make_int4(o[4], o[5], o[6], o[7]);
        } else {
            bad = true;
#pragma unroll
            for (int k = 0; k < 8; ++k)
                if (ok[k])
                    p.dst[8 * i + k] = o[k];
        }
    }
    for (long long i = nvec * 8 + tid; i < p.count; i += stride) {
        int32_t o;
        if (symbol_of(__half2float(p.src[i]), o))
            p.dst[i] = o;
        else
            bad = true;
    }
    if (bad)
        atomicOr(p.out_of_range, 1u);
}

// ------------------------------------------------------------ codec I/O
// YUV420 frame -> model input tensor (reference: prepare_model_input,
// core/src/yuv.cpp:339-400).  One thread per tensor element; the 256-entry
// byte -> FP16 table is built per block in shared memory with the
// reference's arithmetic ((s / 255) * pixel_range in FP32, one rounding).
extern "C" __global__ void __launch_bounds__(256) mlvc_yuv420_to_tensor_f16(const __grid_constant__ YuvParams p)
{
    __shared__ mlvc_half lut[256];
    pdl_launch_dependents();
    lut[threadIdx.x] = __float2half_rn(__fmul_rn(__fdiv_rn(static_cast<float>(threadIdx.x), 255.0f), p.pixel_range));
    __syncthreads();
    pdl_wait();
    const long long plane = static_cast<long long>(p.model_width) * p.model_height;
    const long long total = plane * 3;
    const size_t y_size = static_cast<size_t>(p.width) * p.height;
    const int uv_width = p.width / 2;
    // canvas extent covered by the (possibly transposed) frame
    const int active_w = p.rotated ? p.height : p.width;
    const int active_h = p.rotated ? p.width : p.height;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int ch = static_cast<int>(i / plane);
        const long long s = i - ch * plane;
        const int y = static_cast<int>(s / p.model_width), x = static_cast<int>(s % p.model_width);
        const int cy = min(y, active_h - 1), cx = min(x, active_w - 1);  // edge replication
        const int sy = p.rotated ? cx : cy, sx = p.rotated ? cy : cx;    // frame coordinates
        uint8_t v;
        if (ch == 0)
            v = p.yuv_in[static_cast<size_t>(sy) * p.width + sx];
        else
            v = p.yuv_in[y_size + static_cast<size_t>(ch - 1) * (y_size / 4) + static_cast<size_t>(sy / 2) * uv_width +
                         sx / 2];
        p.t_out[i] = lut[v];
    }
}

__device__ __forceinline__ uint8_t quantize_byte(float v)
{
    v = fminf(fmaxf(v, 0.0f), 1.0f);
    return static_cast<uint8_t>(__float2int_rn(__fmul_rn(v, 255.0f)));
}

// Model output tensor -> YUV420 frame (reference: prepare_model_output_into,
// core/src/yuv.cpp:410-525; values divided by pixel_range in FP32 as there).
// One thread per luma byte; threads of the first quarter also write one U and
// one V byte.
extern "C" __global__ void __launch_bounds__(256) mlvc_tensor_to_yuv420(const __grid_constant__ YuvParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const long long plane = static_cast<long long>(p.model_width) * p.model_height;
    const int y_count = p.width * p.height;
    const int uv_width = p.width / 2, uv_count = y_count / 4;
    auto sample = [&](int ch, int y, int x) {
        const int my = (p.rotated ? x : y) + p.pad_top, mx = (p.rotated ? y : x) + p.pad_left;
        return __fdiv_rn(__half2float(p.t_in[ch * plane + static_cast<long long>(my) * p.model_width + mx]),
                         p.pixel_range);
    };
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < y_count; i += gridDim.x * blockDim.x) {
        const int y = i / p.width, x = i - (i / p.width) * p.width;
        p.yuv_out[i] = quantize_byte(sample(0, y, x));
        if (i < uv_count) {
            const int uy = i / uv_width, ux = i - uy * uv_width;
            float u = __fadd_rn(sample(1, 2 * uy, 2 * ux), sample(1, 2 * uy, 2 * ux + 1));
            float v = __fadd_rn(sample(2, 2 * uy, 2 * ux), sample(2, 2 * uy, 2 * ux + 1));
            u = __fadd_rn(__fadd_rn(u, sample(1, 2 * uy + 1, 2 * ux)), sample(1, 2 * uy + 1, 2 * ux + 1));
            v = __fadd_rn(__fadd_rn(v, sample(2, 2 * uy + 1, 2 * ux)), sample(2, 2 * uy + 1, 2 * ux + 1));
            p.yuv_out[y_count + i] = quantize_byte(__fmul_rn(u, 0.25f));
            p.yuv_out[y_count + uv_count + i] = quantize_byte(__fmul_rn(v, 0.25f));
        }
    }
}

// Model output -> YUV420 straight from the NHWC tensor that the output
// boundary turns into x_hat with an x8 pixel shuffle (3 x 64 channels per
// 1/8-scale pixel; channel c * 64 + dy * 8 + dx is x_hat[c][8 y + dy][8 x + dx]),
// so in the codec's slot path x_hat is never written.  Used when the frame is
// not rotated and its size and position on the canvas are multiples of 8.
// Every sample takes mlvc_tensor_to_yuv420's arithmetic (FP32 division by
// pixel_range, the same order of the chroma sums), so the bytes are the same.
// One thread per 1/8-scale pixel and row dy: 8 luma bytes (one 16-byte load,
// one 8-byte store) and, for even dy, 4 U and 4 V bytes from rows dy, dy + 1.
extern "C" __global__ void __launch_bounds__(256) mlvc_nhwc8_to_yuv420(const __grid_constant__ YuvParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const int fw8 = p.width / 8, fh8 = p.height / 8, mw8 = p.model_width / 8;
    const int total = fw8 * fh8 * 8;
    const int y_count = p.width * p.height, uv_width = p.width / 2, uv_count = y_count / 4;
    const float pr = p.pixel_range;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const int dy = t & 7, q = t >> 3;
        const int fy8 = q / fw8, fx8 = q - fy8 * fw8;
        const mlvc_half* base =
            p.t_in + (static_cast<size_t>(fy8 + p.pad_top / 8) * mw8 + fx8 + p.pad_left / 8) * 192;
        {
            const uint4 v = *reinterpret_cast<const uint4*>(base + dy * 8);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
            uint32_t lo = 0, hi = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float a, b;
                unpack_h2(w[k], a, b);
                const uint32_t pair = quantize_byte(__fdiv_rn(a, pr)) | (quantize_byte(__fdiv_rn(b, pr)) << 8);
                if (k < 2)
                    lo |= pair << (16 * k);
                else
                    hi |= pair << (16 * (k - 2));
            }
            *reinterpret_cast<uint2*>(p.yuv_out + static_cast<size_t>(fy8 * 8 + dy) * p.width + fx8 * 8) =
                make_uint2(lo, hi);
        }
        if (dy & 1)
            continue;
#pragma unroll
        for (int ch = 1; ch <= 2; ++ch) {
            const uint4 r0 = *reinterpret_cast<const uint4*>(base + ch * 64 + dy * 8);
            const uint4 r1 = *reinterpret_cast<const uint4*>(base + ch * 64 + dy * 8 + 8);
            const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w}, w1[4] = {r1.x, r1.y, r1.z, r1.w};
            uint32_t out = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // chroma column 4 fx8 + j: luma columns 2j, 2j + 1
                float a0, b0, a1, b1;
                unpack_h2(w0[j], a0, b0);
                unpack_h2(w1[j], a1, b1);
                float s = __fadd_rn(__fdiv_rn(a0, pr), __fdiv_rn(b0, pr));
                s = __fadd_rn(__fadd_rn(s, __fdiv_rn(a1, pr)), __fdiv_rn(b1, pr));
                out |= static_cast<uint32_t>(quantize_byte(__fmul_rn(s, 0.25f))) << (8 * j);
            }
            *reinterpret_cast<uint32_t*>(p.yuv_out + y_count + (ch - 1) * uv_count +
                                         static_cast<size_t>(fy8 * 4 + dy / 2) * uv_width + fx8 * 4) = out;
        }
    }
}

extern "C" __global__ void __launch_bounds__(256) mlvc_boundary_f16(const __grid_constant__ BoundaryParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ __align__(16) uint8_t dyn_smem[];
    mlvc_half* tile = reinterpret_cast<mlvc_half*>(dyn_smem);
    const bool vec = (p.w * p.r) % 8 == 0 && p.c % 8 == 0;
    if (vec && p.r == 1)
        boundary_vec<1>(p, tile);
    else if (vec && p.r == 2)
        boundary_vec<2>(p, tile);
    else if (vec && p.r == 4)
        boundary_vec<4>(p, tile);
    else if (vec && p.r == 8)
        boundary_vec<8>(p, tile);
    else
        boundary_scalar(p, tile);
}

extern "C" __global__ void mlvc_gather_rows_f16(const __grid_constant__ GatherParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    int row = p.index[0];
    if (row < 0)
        row += p.rows;
    if (row < 0 || row >= p.rows) {
        // the reference CPU backend raises "GATHER index out of range"
        // (backends/cpu/src/execution_plan.cpp:119-124); here the run reports it
        if (blockIdx.x == 0 && threadIdx.x == 0)
            atomicOr(&mlvc_b200_status, mlvc_b200::kStatusGatherIndex);
        return;
    }
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < p.row_elems; i += stride)
        p.dst[i] = p.src[row * p.row_elems + i];
}

// --------------------------------------------------------- pixel ops
// DepthToSpace (CRD, PyTorch pixel_shuffle) on NHWC: output pixel (y, x)
// channel c reads input pixel (y / r, x / r) channel c*r*r + (y%r)*r + x%r.
extern "C" __global__ void mlvc_depth_to_space_f16(const __grid_constant__ PixelShuffleParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const int r = p.r, oc = p.c / (r * r), ow = p.w * r, oh = p.h * r;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < p.count; i += stride) {
        long long t = i;
        const int c = static_cast<int>(t % oc);
        t /= oc;
        const int x = static_cast<int>(t % ow);
        t /= ow;
        const int y = static_cast<int>(t % oh);
        const long long n = t / oh;
        const int ic = c * r * r + (y % r) * r + (x % r);
        p.dst[i] = p.src[((n * p.h + y / r) * p.w + x / r) * p.c + ic];
    }
}

// DepthToSpace with r = 2, output channels a multiple of 8: one thread per
// input pixel and 8 output channels (4 x 16-byte loads of 32 input channels,
// 4 x 16-byte stores, one per output sub-pixel s = dy * 2 + dx, which takes
// input channels 4 j + s).  `count` = input pixels x output channels / 8.
template <typename I>
__device__ __forceinline__ void depth_to_space_r2_v8(const PixelShuffleParams& p)
{
    const I ocv = p.c / 32;  // 8-channel output blocks per pixel
    const I w = p.w, ow = w * 2;
    const I count = static_cast<I>(p.count);
    const I stride = static_cast<I>(gridDim.x) * blockDim.x;
    for (I i = static_cast<I>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
        const I m = i % ocv;
        const I px = i / ocv;  // input pixel (n, y, x)
        const I x = px % w;
        const I ny = px / w;  // n * h + y
        const uint4* src = reinterpret_cast<const uint4*>(p.src + static_cast<size_t>(px) * p.c + m * 32);
        uint32_t wv[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 v = src[q];
            wv[4 * q] = v.x;
            wv[4 * q + 1] = v.y;
            wv[4 * q + 2] = v.z;
            wv[4 * q + 3] = v.w;
        }
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const int dy = s >> 1, dx = s & 1;
            const uint32_t sel = (s & 1) ? 0x7632u : 0x5410u;  // high or low halves
            uint32_t o[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
                o[k] = __byte_perm(wv[4 * k + (s >> 1)], wv[4 * k + 2 + (s >> 1)], sel);
            const size_t orow = (static_cast<size_t>(ny) * 2 + dy) * ow + 2 * x + dx;  // output pixel (n, 2y + dy, 2x + dx)
            *reinterpret_cast<uint4*>(p.dst + orow * (p.c / 4) + m * 8) = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

extern "C" __global__ void __launch_bounds__(256) mlvc_depth_to_space_r2_v8_f16(const __grid_constant__ PixelShuffleParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    if (p.count < (1ll << 31))
        depth_to_space_r2_v8<unsigned>(p);
    else
        depth_to_space_r2_v8<long long>(p);
}

// SpaceToDepth with r = 2, input channels a multiple of 8: one thread per
// output pixel and 8 input channels (the inverse of the kernel above).
// `count` = output pixels x input channels / 8.
extern "C" __global__ void __launch_bounds__(256) mlvc_space_to_depth_r2_v8_f16(const __grid_constant__ PixelShuffleParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const int icv = p.c / 8;
    const int ow = p.w / 2;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < p.count; i += stride) {
        const int m = static_cast<int>(i % icv);
        const long long opx = i / icv;  // output pixel (n, y, x)
        const int x = static_cast<int>(opx % ow);
        const long long ny = opx / ow;
        uint32_t v[4][4];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const int dy = s >> 1, dx = s & 1;
            const long long irow = (ny * 2 + dy) * p.w + 2 * x + dx;
            const uint4 u = *reinterpret_cast<const uint4*>(p.src + irow * p.c + m * 8);
            v[s][0] = u.x;
            v[s][1] = u.y;
            v[s][2] = u.z;
            v[s][3] = u.w;
        }
        // output channel 4 j + s of block m <- input channel j of sub-pixel s
        uint4* dst = reinterpret_cast<uint4*>(p.dst + opx * (p.c * 4) + m * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // output channels 8 q .. 8 q + 7 of the block: j = 2 q, 2 q + 1
            uint32_t o[4];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const int j = 2 * q + t;
                const uint32_t sel = (j & 1) ? 0x7632u : 0x5410u;
                o[2 * t] = __byte_perm(v[0][j >> 1], v[1][j >> 1], sel);
                o[2 * t + 1] = __byte_perm(v[2][j >> 1], v[3][j >> 1], sel);
            }
            dst[q] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

// SpaceToDepth (PyTorch pixel_unshuffle) on NHWC: output channel
// c*r*r + dy*r + dx of pixel (y, x) reads input pixel (y*r+dy, x*r+dx) channel c.
extern "C" __global__ void mlvc_space_to_depth_f16(const __grid_constant__ PixelShuffleParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const int r = p.r, oh = p.h / r, ow = p.w / r, oc = p.c * r * r;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < p.count; i += stride) {
        long long t = i;
        const int c = static_cast<int>(t % oc);
        t /= oc;
        const int x = static_cast<int>(t % ow);
        t /= ow;
        const int y = static_cast<int>(t % oh);
        const long long n = t / oh;
        const int ic = c / (r * r), off = c % (r * r);
        p.dst[i] = p.src[((n * p.h + y * r + off / r) * p.w + x * r + off % r) * p.c + ic];
    }
}

// ------------------------------------------------------------- ReGLU
extern "C" __global__ void mlvc_reglu_f16(const __grid_constant__ RegluParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const long long total = p.pixels * p.c;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total; i += stride) {
        const long long px = i / p.c;
        const int c = static_cast<int>(i % p.c);
        const float g = __half2float(p.src[px * 2 * p.c + c]);
        const float l = __half2float(p.src[px * 2 * p.c + p.c + c]);
        const float cg = round_h(fminf(fmaxf(g, p.lo), p.hi));
        p.dst[i] = __float2half_rn(cg * l);
    }
}

// --------------------------------------------------------- depthwise
// One thread produces 8 consecutive channels of one output pixel (16-byte
// loads of input and weights); weights are [kh*kw][C].  Requires C % 8 == 0.
extern "C" __global__ void mlvc_depthwise_v8_f16(const __grid_constant__ DirectConvParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const int cv = p.oc / 8;
    const long long total = static_cast<long long>(p.n) * p.oh * p.ow * cv;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total; i += stride) {
        long long t = i;
        const int c8 = static_cast<int>(t % cv) * 8;
        t /= cv;
        const int ox = static_cast<int>(t % p.ow);
        t /= p.ow;
        const int oy = static_cast<int>(t % p.oh);
        const long long n = t / p.oh;
        float acc[8];
        if (p.bias) {
            const uint4 bv = *reinterpret_cast<const uint4*>(p.bias + c8);
            const uint32_t* bw = reinterpret_cast<const uint32_t*>(&bv);
#pragma unroll
            for (int k = 0; k < 4; ++k)
                unpack_h2(bw[k], acc[2 * k], acc[2 * k + 1]);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k)
                acc[k] = 0.0f;
        }
        for (int ky = 0; ky < p.kh; ++ky) {
            const int iy = oy * p.sh + ky - p.ph;
            if (iy < 0 || iy >= p.ih)
                continue;
            for (int kx = 0; kx < p.kw; ++kx) {
                const int ix = ox * p.sw + kx - p.pw;
                if (ix < 0 || ix >= p.iw)
                    continue;
                const uint4 xv = *reinterpret_cast<const uint4*>(p.x + ((n * p.ih + iy) * p.iw + ix) * p.ic + c8);
                const uint4 wv = *reinterpret_cast<const uint4*>(p.w + (ky * p.kw + kx) * p.oc + c8);
                const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv);
                const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    float x0, x1, w0, w1;
                    unpack_h2(xw[k], x0, x1);
                    unpack_h2(ww[k], w0, w1);
                    acc[2 * k] = fmaf(x0, w0, acc[2 * k]);
                    acc[2 * k + 1] = fmaf(x1, w1, acc[2 * k + 1]);
                }
            }
        }
        uint4 ov;
        uint32_t* o = reinterpret_cast<uint32_t*>(&ov);
#pragma unroll
        for (int k = 0; k < 4; ++k)
            o[k] = pack_h2(acc[2 * k], acc[2 * k + 1]);
        *reinterpret_cast<uint4*>(p.y + i * 8) = ov;
    }
}

// Depthwise 3x3 (stride 1 or 2, pad 0 or 1), specialised: each thread owns 8
// consecutive channels (16 bytes) of kRows vertically adjacent output pixels.
// A block of 256 threads covers 256 / (C/8) adjacent output columns of one
// row strip (grid: x = column groups, y = row strips, z = images), so the
// index math is 32-bit and division-free.  The thread walks the three kernel
// columns; per column it loads the (kRows-1)*stride+3 input vectors it needs
// (all in flight together), converts each input and each weight to FP32
// exactly once and feeds every output row that uses it, so conversions stay
// well below the FMA count.  The accumulation starts from the bias with FP32
// FMA; taps that fall outside the image contribute nothing.
template <int kStride>
__device__ __forceinline__ void depthwise3x3_body(const DirectConvParams& p)
{
    constexpr int kRows = 4;
    constexpr int kInRows = (kRows - 1) * kStride + 3;
    const int cv = p.oc / 8;
    const int per_block = blockDim.x / cv;
    const int c8 = (threadIdx.x % cv) * 8;
    const int ox = blockIdx.x * per_block + threadIdx.x / cv;
    if (threadIdx.x >= per_block * cv || ox >= p.ow)
        return;
    const int oy0 = blockIdx.y * kRows;
    const int n = blockIdx.z;
    const int iy0 = oy0 * kStride - p.ph, ix0 = ox * kStride - p.pw;
    const mlvc_half* xin = p.x + static_cast<size_t>(n) * p.ih * p.iw * p.ic + c8;
    float acc[kRows][8];
    {
        float bias[8];
        if (p.bias) {
            const uint4 bv = __ldg(reinterpret_cast<const uint4*>(p.bias + c8));
            const uint32_t* bw = reinterpret_cast<const uint32_t*>(&bv);
#pragma unroll
            for (int k = 0; k < 4; ++k)
                unpack_h2(bw[k], bias[2 * k], bias[2 * k + 1]);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k)
                bias[k] = 0.0f;
        }
#pragma unroll
        for (int r = 0; r < kRows; ++r)
#pragma unroll
            for (int k = 0; k < 8; ++k)
                acc[r][k] = bias[k];
    }
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
        const int ix = ix0 + kx;
        if (ix < 0 || ix >= p.iw)
            continue;
        uint4 col[kInRows];
#pragma unroll
        for (int j = 0; j < kInRows; ++j) {
            const int iy = iy0 + j;
            col[j] = (iy >= 0 && iy < p.ih)
                         ? *reinterpret_cast<const uint4*>(xin + (static_cast<size_t>(iy) * p.iw + ix) * p.ic)
                         : make_uint4(0, 0, 0, 0);
        }
        float w[3][8];
#pragma unroll
        for (int ky = 0; ky < 3; ++ky) {
            const uint4 wv = __ldg(reinterpret_cast<const uint4*>(p.w + (ky * 3 + kx) * p.oc + c8));
            const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
#pragma unroll
            for (int k = 0; k < 4; ++k)
                unpack_h2(ww[k], w[ky][2 * k], w[ky][2 * k + 1]);
        }
#pragma unroll
        for (int j = 0; j < kInRows; ++j) {
            float xf[8];
            const uint32_t* xw = reinterpret_cast<const uint32_t*>(&col[j]);
#pragma unroll
            for (int k = 0; k < 4; ++k)
                unpack_h2(xw[k], xf[2 * k], xf[2 * k + 1]);
#pragma unroll
            for (int r = 0; r < kRows; ++r) {
                const int ky = j - r * kStride;
                if (ky < 0 || ky > 2)
                    continue;
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    acc[r][k] = fmaf(xf[k], w[ky][k], acc[r][k]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
        const int oy = oy0 + r;
        if (oy >= p.oh)
            break;
        uint4 ov;
        uint32_t* o = reinterpret_cast<uint32_t*>(&ov);
#pragma unroll
        for (int k = 0; k < 4; ++k)
            o[k] = pack_h2(acc[r][2 * k], acc[r][2 * k + 1]);
        *reinterpret_cast<uint4*>(p.y + ((static_cast<size_t>(n) * p.oh + oy) * p.ow + ox) * p.oc + c8) = ov;
    }
}

extern "C" __global__ void __launch_bounds__(256, 2) mlvc_depthwise3x3_f16(const __grid_constant__ DirectConvParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    if (p.sh == 2)
        depthwise3x3_body<2>(p);
    else
        depthwise3x3_body<1>(p);
}

// Generic grouped direct convolution (fallback for shapes the tensor-core
// kernels do not cover).  Weights are [OC][kh][kw][ICg]; optional fused
// LeakyReLU / residual with the graph's double rounding.
extern "C" __global__ void mlvc_conv_direct_f16(const __grid_constant__ DirectConvParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const long long total = static_cast<long long>(p.n) * p.oh * p.ow * p.oc;
    const int icg = p.ic / p.groups, ocg = p.oc / p.groups;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total; i += stride) {
        long long t = i;
        const int o = static_cast<int>(t % p.oc);
        t /= p.oc;
        const int ox = static_cast<int>(t % p.ow);
        t /= p.ow;
        const int oy = static_cast<int>(t % p.oh);
        const long long n = t / p.oh;
        const int g = o / ocg;
        float acc = p.bias ? __half2float(p.bias[o]) : 0.0f;
        for (int ky = 0; ky < p.kh; ++ky) {
            const int iy = oy * p.sh + ky - p.ph;
            if (iy < 0 || iy >= p.ih)
                continue;
            for (int kx = 0; kx < p.kw; ++kx) {
                const int ix = ox * p.sw + kx - p.pw;
                if (ix < 0 || ix >= p.iw)
                    continue;
                const mlvc_half* xr = p.x + ((n * p.ih + iy) * p.iw + ix) * p.ic + g * icg;
                const mlvc_half* wr = p.w + ((static_cast<long long>(o) * p.kh + ky) * p.kw + kx) * icg;
                for (int c = 0; c < icg; ++c)
                    acc = fmaf(__half2float(xr[c]), __half2float(wr[c]), acc);
            }
        }
        float v = round_h(acc);
        if (p.epilogue == kEpiLeaky)
            v = v < 0.0f ? round_h(v * p.alpha) : v;
        else if (p.epilogue == kEpiResidual)
            v = v + __half2float(p.residual[i]);
        p.y[i] = __float2half_rn(v);
    }
}

}  // namespace mlvc_b200
