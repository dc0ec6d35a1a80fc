// Kernel parameter blocks shared by the host runtime (C++) and the sm_100a
// kernels.  Every kernel takes exactly one of these structs by value
// (`const __grid_constant__`), so the host launches it with a single
// kernelParams entry and CUDA-graph capture copies it once.
#pragma once

#include <cuda.h>
#include <stdint.h>

#ifdef __CUDACC__
#include <cuda_fp16.h>
typedef __half mlvc_half;
#else
typedef uint16_t mlvc_half;
#endif

namespace mlvc_b200 {

// Shared-memory bytes reserved at the start of a tensor-core conv CTA for
// barriers, the TMEM address and the bias slice (operand tiles follow,
// 1024-byte aligned).
constexpr int kTcHeaderBytes = 2048;

// Epilogue staging of a tensor-core conv CTA: the whole output tile, 128 rows
// x 128 bytes per 64 output columns (128-byte swizzle), stored by TMA.
constexpr int kTcStagePanelBytes = 128 * 128;

// Epilogue kinds of the tensor-core conv kernels.  Rounding follows the graph:
// the conv result is rounded to FP16 first, then the fused operator is applied
// and rounded again.
enum Epilogue : int {
    kEpiBias = 0,      // y = fp16(acc + bias)
    kEpiLeaky = 1,     // y = leaky(fp16(acc + bias))
    kEpiResidual = 2,  // y = fp16(fp16(acc + bias) + r)
    kEpiReglu = 3,     // columns [0, BN/2) gate, [BN/2, BN) linear of the same channels
};

// Shared by the 1x1 GEMM and the k x k implicit-GEMM conv kernels.
struct ConvTcParams {
    CUtensorMap map_a0;  // activations (1x1: [M rows, K]; kxk: parity 0 view)
    CUtensorMap map_a1;  // kxk stride-2: parity 1 view (unused otherwise)
    CUtensorMap map_b;   // prepared weights [N rows, K = taps * IC] (K-major)
    // Output store view and residual load view (same geometry): 1x1 {channels,
    // pixels} with {64, 128} boxes, kxk {channels, W, H} with {64, 128, 1}
    // boxes, 128-byte swizzle; stores and loads are clipped / zero-filled at the
    // tensor edges, so partial tiles need no special case.
    CUtensorMap map_out;
    CUtensorMap map_res;
    const mlvc_half* bias;      // [N] in prepared column order, may be null
    mlvc_half* out;             // NHWC output (written through map_out; kept for debugging)
    int M, N, K;                // GEMM extents (K = taps * IC); N counts prepared (padded) weight rows
    int n_valid;                // output channels actually stored (<= N)
    int BN;                     // columns per N tile (multiple of 64, <= 256; ReGLU: multiple of 128)
    int n_tiles, m_tiles;       // tile counts
    int epilogue;               // Epilogue
    float alpha, clip_lo, clip_hi;
    int a_stages;               // A ring depth (1x1: 16 KB panels; kxk: halo blocks)
    int b_resident;             // kxk: 1 = all weight panels resident in smem
    int b_stages;               // kxk: B ring depth when not resident
    // kxk geometry (ignored by the 1x1 kernel)
    int in_h, in_w, in_c;
    int out_h, out_w;
    int kh, kw, stride, pad;
    int halo_px;                // pixels (or pixel pairs) per halo row
    int px_min;                 // leftmost halo offset relative to the tile start (<= 0)
    int a_split;                // 1x1: K panels from this index on come from map_a1 (a channel concat of two
                                // tensors read in place); 0: all from map_a0
    int stage_bufs;             // 1x1 / k x k: output staging buffers (2: a tile's rows are written while the
                                // previous tile's TMA store still reads the other buffer; 0 or 1: one)
    // Optional phase trace (null in normal runs): kTracePoints %globaltimer
    // stamps per CTA, written by the role that reaches each point.
    unsigned long long* trace;
    // Wait-expiry test only (0 in every normal launch): k > 0 makes CTA 0's
    // producer leave its k-th A panel unloaded -- no TMA is issued and the
    // stage's barrier is never armed -- so the MMA issuer's bounded wait for
    // it runs out and the CTA takes its abort path.  1x1 kernel only.
    int withhold_a;
    // 1x1 with a pixel shuffle (r = 2) after it, folded into the store: the
    // tiles are row-aligned (row_tiles per input row of in_w pixels, in_h
    // rows), weight rows are ordered [sub-pixel dy * 2 + dx][channel], and
    // map_out is the 5-D view {C, dx, x, dy, y} of the [2 in_h, 2 in_w, C]
    // output with C = d2s_c.  0 / 0: linear pixel tiles, 2-D output map.
    int d2s_c;
    int row_tiles;
};

// Phase trace points of the tensor-core conv kernels.
enum TracePoint : int {
    kTrEntry = 0,          // CTA start
    kTrSetup = 1,          // barriers initialised, TMEM allocated
    kTrWeightsIssued = 2,  // producer issued the weight loads
    kTrWeightsLanded = 3,  // MMA issuer saw the weights arrive
    kTrFirstA = 4,         // MMA issuer saw the first activation panel
    kTrLastCommit = 5,     // MMA issuer committed its last tile
    kTrFirstAcc = 6,       // epilogue saw the first accumulator
    kTrEpilogueDone = 7,   // epilogue finished its last tile
    kTrExit = 8,           // CTA teardown done
    kTrFfnHidden0 = 9,     // fused FFN: epilogue wrote the first hidden chunk
    kTrFfnHiddenLast = 10, // fused FFN: epilogue wrote the first tile's last hidden chunk
    kTrFfnAcc2 = 11,       // fused FFN: epilogue saw the first tile's output accumulator
    kTrFfnXIssued = 12,    // fused FFN: producer issued the first X tile
    kTrFfnChunkWaited = 13,  // fused FFN: epilogue passed both waits of hidden chunk 1
    kTrFfnChunkLoaded = 14,  // fused FFN: chunk 1 accumulators in registers
    kTrFfnChunkStored = 15,  // fused FFN: chunk 1 written to shared memory
    kTrFfnG1First = 16,      // fused FFN: MMA issuer committed GEMM1 of chunk 0
    kTrFfnG1Second = 17,     // fused FFN: MMA issuer committed GEMM1 of chunk 1
    kTrFfnG2First = 18,      // fused FFN: MMA issuer passed the waits of GEMM2 chunk 0
    kTrFfnChunk1Done = 19,   // fused FFN: epilogue released hidden chunk 1
    kTrDwFirstSlice = 20,    // fused depthwise (+ expand): first depthwise slice written as an A panel
    kTrDepReady = 21,        // producer's griddepcontrol.wait returned: the previous kernel's outputs are visible
    // fused block, first tile, expand chunk c < 4: compute leader saw the expand
    // accumulator (kTrMbChunk + 3c), the chunk complete in shared memory
    // (+1), its A panel written (+2); MMA issuer passed the waits of the expand
    // GEMM (kTrMbExpandMma + c) and of the projection K slice (kTrMbProjMma + c)
    kTrMbChunk = 24,
    kTrMbExpandMma = 36,
    kTrMbProjMma = 40,
    // fused depthwise (mlvc_dwconv_tc), first tile, slice s < 8: A panel
    // written (kTrDwSlice + s), MMA issuer passed its waits (kTrDwMma + s);
    // second tile's first slice written (kTrDwTile1)
    kTrDwSlice = 24,
    kTrDwTile1 = 32,
    kTrDwMma = 36,
    // 1x1 / k x k conv, the CTA's tiles i < 4: MMA issuer began the tile
    // (accumulator free: kTrConvTile + 4i), committed it (+1), the epilogue
    // finished it (stores issued, +2); epilogue leader saw the accumulator
    // (kTrConvEpi + 4i), the staging buffer ready (+1), wrote its rows (+2),
    // saw every row written (+3)
    kTrConvEpi = 24,
    kTrConvTile = 48,
    kTracePoints = 64
};

// Fused feed-forward block (mlvc_ffn_tc):
//     hidden = clip(fp16(X W1g^T + b1g), lo, hi) * fp16(X W1l^T + b1l)   (ReGLU, FP16 rounding per op)
//     out    = epilogue(fp16(hidden W2^T + b2))                           (bias / LeakyReLU / + residual)
// The hidden tensor stays in shared memory, 64 channels at a time.
constexpr int kFfnHeaderBytes = 4096;  // barriers, TMEM address, both bias vectors
constexpr int kFfnChunk = 64;          // hidden channels per chunk
constexpr int kFfnMaxHidden = 256;     // bias1 capacity in the header (2 x hidden floats)
constexpr int kFfnMaxWStages = 12;     // weight ring slots (barrier pairs in the header)

struct FfnTcParams {
    // map_a0 = X [M, C] (128 x 64 boxes), map_b = W1 in chunk order
    // [hidden/64 x (64 gate + 64 linear) rows, C] (128 x 64 boxes), map_out /
    // bias (b2) / residual / out / epilogue describe the second conv's output;
    // K = C, BN = N = n_valid = output channels, a_stages = X tiles in flight,
    // b_stages = weight ring slots, clip_lo/clip_hi = ReGLU clip.
    ConvTcParams c;
    CUtensorMap map_w2;      // W2 [C_out rows, hidden] (C_out x 64 boxes)
    const mlvc_half* bias1;  // [2 x hidden] in W1's chunk order
    int hidden;              // hidden channels (multiple of 64, <= kFfnMaxHidden)
    int w_slot_bytes;        // bytes per weight ring slot (max of a W1 and a W2 panel)
    // Shared memory: header, X tiles (a_stages), two hidden panels (also the
    // output epilogue's staging buffers), weight ring (b_stages slots).
};

// Fused depthwise 3x3 (stride 1, pad 1) + 1x1 conv (mlvc_dwconv_tc):
//     d   = fp16(dw3x3(x) + b_dw)               CUDA cores, FP32 FMA from the bias
//     out = epilogue(fp16(d W^T + b))           tcgen05; bias / LeakyReLU / + residual
// The depthwise result of each 16 x 8-pixel tile is written straight into the
// GEMM's A operand in shared memory, 64 channels at a time.
constexpr int kDwHeaderBytes = 2048;
constexpr int kDwTileW = 16, kDwTileH = 8;                        // output tile (pixels)
constexpr int kDwHaloPx = (kDwTileW + 2) * (kDwTileH + 2);        // 180 halo pixels per slice
constexpr int kDwHaloBytes = (kDwHaloPx * 128 + 1023) / 1024 * 1024;  // one 64-channel halo slice in smem
// Fused depthwise CTA: TMA warp, MMA warp, 8 depthwise warps, then 4 output
// epilogue warps (one per TMEM lane quadrant) that drain tile t's accumulator
// while the depthwise warps compute tile t + 1.
constexpr int kDwComputeThreads = 256;
constexpr int kDwEpilogueThreads = 128;
constexpr int kDwThreads = 64 + kDwComputeThreads + kDwEpilogueThreads;

// Channels per depthwise-taps TMA box of mlvc_dwconv_tc: the largest multiple
// of 64 that is at most 256 (a box dimension limit) and divides C, so the
// boxes tile [10][C] exactly (C a multiple of 64).
#ifdef __CUDACC__
__host__ __device__
#endif
inline int dw_tap_group(int c)
{
    for (int t = 256; t >= 64; t -= 64)
        if (c % t == 0)
            return t;
    return 64;
}

struct DwConvTcParams {
    // map_b = W [C_out rows, C] (C_out x 64 boxes, 128-byte swizzle);
    // map_out / map_res / bias / epilogue / alpha describe the 1x1 conv's
    // output; K = C, BN = N = n_valid = C_out, a_stages = A panels in flight,
    // b_stages = W ring slots.
    ConvTcParams c;
    // Tiles are kDwTileW x kDwTileH pixels (128 = one MMA tile); map_out /
    // map_res use {64, kDwTileW, kDwTileH} boxes over {C_out, W, H}.
    CUtensorMap map_halo;    // x {C, W, H} in {64, kDwTileW + 2, kDwTileH + 2} boxes, no swizzle (128-byte pixel rows)
    CUtensorMap map_dw;      // depthwise taps and bias [10][C] (rows 0..8: tap ky * 3 + kx, row 9: bias), one {C, 10} box
    int width, height;       // image
    int tiles_x;             // tiles per image row
    int h_stages;            // halo slices in flight (1 or 2)
};

// Fused inverted-residual block (mlvc_mbconv_tc):
//     e   = epi1(fp16(x W1^T + b1))             tcgen05 over the 18 x 10 halo; bias (+ LeakyReLU),
//                                               zero outside the image (the depthwise padding)
//     d   = fp16(dw3x3(e) + b_dw)               CUDA cores, FP32 FMA from the bias
//     out = epilogue(fp16(d W2^T + b2))         tcgen05; bias / LeakyReLU / + residual
// Per 16 x 8-pixel tile the expanded tensor e exists only in shared memory,
// 64 channels at a time.
constexpr int kMbHeaderBytes = 4096;                              // barriers, TMEM address, both bias vectors
constexpr int kMbMaxExpand = 256;                                 // expanded channels (bias1 capacity)
constexpr int kMbHaloRows = 184;                                  // 180 halo pixels, padded to whole 8-row swizzle atoms
constexpr int kMbSliceBytes = kMbHaloRows * 128;                  // one 64-channel halo slice (x or e) in smem
constexpr int kMbRow1 = 56;                                       // first halo row of the second GEMM1 M block (rows 56..183)
constexpr int kMbWSlotBytes = 16384;                              // one weight ring slot
constexpr int kMbWStages = 3;
constexpr int kMbBlockThreads = 576;                              // TMA warp, MMA warp, 16 compute warps

struct MbConvTcParams {
    // c describes the projection conv (as for mlvc_dwconv_tc): map_b = W2
    // [C_out rows, E] (C_out x 64 boxes, 128-byte swizzle), map_out / map_res
    // in {64, 16, 8} boxes over {C_out, W, H}, bias = b2, epilogue / alpha =
    // its fused operator, K = E, BN = N = n_valid = C_out, m_tiles = tiles.
    ConvTcParams c;
    CUtensorMap map_x;       // x {C, W, H} in {64, 18, 10} boxes, 128-byte swizzle (GEMM1's A operand)
    CUtensorMap map_w1;      // W1 [E rows, C] in {64, 64} boxes, 128-byte swizzle
    CUtensorMap map_dw;      // depthwise taps and bias [10][E] (rows 0..8: tap ky * 3 + kx, row 9: bias), one {E, 10} box
    const mlvc_half* bias1;  // [E] expand bias
    float alpha1;            // expand LeakyReLU slope (epi1 == kEpiLeaky)
    int epi1;                // kEpiBias or kEpiLeaky
    int c_in;                // C (multiple of 64, <= 128)
    int expand;              // E (multiple of 64, <= kMbMaxExpand)
    int width, height;       // image
    int tiles_x;             // tiles per image row
};

struct ElementwiseParams {
    const mlvc_half* a;
    const mlvc_half* b;
    mlvc_half* out;
    long long count;    // output elements
    int op;             // unary: 0 leaky 1 clip 2 sigmoid 3 reciprocal 4 round; binary: 0 add 1 mul 2 sub
    float alpha, lo, hi;
    // broadcast binary: output logical dims (n, c, h, w) in physical NHWC order and per-operand strides
    int dims[4];        // n, h, w, c extents of the output (physical order)
    long long sa[4];    // element strides of `a` for (n, h, w, c)
    long long sb[4];
};

// Generic strided copy over up to 4 logical dimensions (physical order of the
// output): slice, concat pieces, layout conversion.
struct CopyParams {
    const mlvc_half* src;
    mlvc_half* dst;
    int dims[4];
    long long ss[4];
    long long ds[4];
    long long count;
};

struct GatherParams {
    const mlvc_half* src;
    const int32_t* index;
    mlvc_half* dst;
    long long row_elems;
    int rows;
};

// Depthwise / generic grouped direct convolution on NHWC tensors.
struct DirectConvParams {
    const mlvc_half* x;
    const mlvc_half* w;     // depthwise: [kh*kw][C]; generic: [OC][kh][kw][ICg]
    const mlvc_half* bias;  // [OC] or null
    const mlvc_half* residual;
    mlvc_half* y;
    int n, ih, iw, ic, oh, ow, oc;
    int kh, kw, sh, sw, ph, pw, groups;
    int epilogue;
    float alpha;
};

struct PixelShuffleParams {
    const mlvc_half* src;
    mlvc_half* dst;
    int n, h, w, c;  // input NHWC extents
    int r;           // block size
    long long count;
};

// Boundary conversion between the host's NCHW and the device's NHWC, fused
// with pixel (un)shuffle by `r` (r = 1: plain layout conversion).  (n, h, w, c)
// are the DEVICE tensor's NHWC extents; the host tensor is NCHW
// [n][c/(r*r)][h*r][w*r].
//   to_host = 0: device <- host, i.e. pixel_unshuffle(r) of the host tensor
//   to_host = 1: host <- device, i.e. pixel_shuffle(r) of the device tensor
struct BoundaryParams {
    const mlvc_half* src;
    mlvc_half* dst;
    int n, h, w, c;
    int r;
    int to_host;
};

struct RegluParams {
    const mlvc_half* src;  // NHWC [P, 2C]
    mlvc_half* dst;        // NHWC [P, C]
    long long pixels;
    int c;
    float lo, hi;
};

// Fused recurrent-feature update (mlvc_feature_update_f16), per element with
// the graph's FP16 rounding after every operator:
//   sb = sigmoid(b), sc = sigmoid(c), blended = sb * history + (one - sb) * a,
//   scaled = (sc * blended) * scale[channel]
// where a, b, c are the three channel thirds of src.  Writes the channel
// concat [scaled, blended] and, where the graph reads them elsewhere, scaled
// and blended on their own (each pointer may be null).
struct FeatureUpdateParams {
    const mlvc_half* src;      // NHWC [P, 3C]
    const mlvc_half* history;  // NHWC [P, C]
    const mlvc_half* scale;    // [C]
    mlvc_half* concat;         // NHWC [P, 2C]
    mlvc_half* scaled;         // NHWC [P, C]
    mlvc_half* blended;        // NHWC [P, C]
    long long pixels;
    int c;                     // channels (multiple of 8)
    float one;                 // the scalar the gate is subtracted from (1 in exported graphs)
};

// Fused latent quantisation tails (mlvc_y0_tail_f16 / mlvc_y1_tail_f16),
// per pixel and channel q < Q with the graph's FP16 rounding after every
// operator (reference: backends/driver_cubin/kernels/quantization_tail.cu and
// the matchers of fusion_registry.cpp:14-404).  Halves j = 0, 1 are channels
// j * Q + q of the 2Q-channel tensors.
//   y0: clipped_j = max(prior[j], lo), normalized_j = latent_j * (1 / clipped_j),
//       s_j = (normalized_j - prior[2Q + j]) * qscale_j, y = round(s_0 + s_1),
//       u_j = (y + prior[2Q + j]) * uscale_j; concat2 = [u_0, u_1],
//       concat3 = [u_0, u_1, prior (4Q)]
//   y1: s_j = (normalized_j - prior_j) * qscale_j, y = round(s_0 + s_1),
//       u_j = (y + prior_j) * uscale_j, result_j = (concat2_j + u_j) * clipped_j
// Side outputs the graph reads elsewhere are written when non-null.
struct QuantTailParams {
    const mlvc_half* latent;      // y0: [P, 2Q]
    const mlvc_half* normalized;  // y1: [P, 2Q]
    const mlvc_half* prior;       // y0: [P, 4Q]; y1: [P, 2Q]
    const mlvc_half* qscale;      // [P, 2Q]
    const mlvc_half* uscale0;     // [P, Q]
    const mlvc_half* uscale1;     // [P, Q]
    const mlvc_half* concat2_in;  // y1: [P, 2Q]
    const mlvc_half* clipped_in;  // y1: [P, 2Q]
    mlvc_half* normalized_out;    // y0 side output [P, 2Q] or null
    mlvc_half* clipped_out;       // y0 side output [P, 2Q] or null
    mlvc_half* y_raw;             // [P, Q]
    mlvc_half* concat2_out;       // y0 side output [P, 2Q] or null
    mlvc_half* concat3;           // y0: [P, 6Q]
    mlvc_half* result;            // y1: [P, 2Q]
    long long pixels;
    int q;                        // Q (multiple of 8)
    float clip_lo;                // y0 clip lower bound
};

// Codec I/O between a YUV420 frame (planar Y, U, V bytes, width x height,
// both even) and the model's [1, 3, model_height, model_width] FP16 NCHW
// tensor, with the reference's conventions (core/src/yuv.cpp:324-525): the
// frame sits at the top-left of the model canvas, transposed when it only
// fits rotated; input pixels are byte * pixel_range / 255 rounded to FP16 and
// replicate the last row / column into the padding; output bytes are
// round(clamp(value / pixel_range, 0, 1) * 255), chroma from the mean of a
// 2x2 block summed in raster order.
// Scale extraction for the entropy coder (mlvc_extract_scales; reference
// extract_scales, core/src/scales.cpp:25-105): z [hyper][zh][zw] FP16 ->
// scales_0 / scales_1 int32 [latent / 2][yh][yw].
struct ScaleParams {
    const mlvc_half* z;
    int32_t* scales_0;
    int32_t* scales_1;
    int z_height, z_width;
    int latent, repeat;      // latent channels, y_scale_repeat
    int y_height, y_width;
    int spatial;             // downsample_hyperprior (nearest up-sampling factor)
    int max_index;           // scale_max_index
    int vec4;                // 1: four outputs per thread (y_width % 4 == 0, planes 16-byte aligned)
};

// FP16 latents -> int32 entropy symbols (mlvc_integer_values_f16; reference
// integer_values, core/src/entropy.cpp:201-226).
struct IntegerValuesParams {
    const mlvc_half* src;
    int32_t* dst;
    long long count;
    unsigned int* out_of_range;  // set to 1 when a value is not finite or outside [-32768, 32767]
    int vec8;                    // 1: src and dst 16-byte aligned (8 values per thread)
};

struct YuvParams {
    const uint8_t* yuv_in;    // to tensor: Y | U | V planes
    uint8_t* yuv_out;         // from tensor
    const mlvc_half* t_in;    // from tensor: NCHW [3, model_height, model_width]
    mlvc_half* t_out;         // to tensor
    int width, height;        // frame
    int model_width, model_height;
    int pad_left, pad_top;    // position of the frame on the canvas (output side)
    int rotated;              // 1: the canvas holds the transposed frame
    float pixel_range;
};

}  // namespace mlvc_b200
