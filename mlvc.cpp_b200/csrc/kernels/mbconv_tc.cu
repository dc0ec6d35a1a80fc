// Fused inverted-residual block for sm_100a (tcgen05 + CUDA cores + TMA):
//
//     e   = epi1(fp16(x W1^T + b1))      1x1 expand conv (+ LeakyReLU), zero outside the image
//     d   = fp16(dw3x3(e) + b_dw)        depthwise 3x3, stride 1, pad 1, FP32 FMA from the bias
//     out = epilogue(fp16(d W2^T + b2))  1x1 projection conv (+ residual / LeakyReLU)
//
// This is the graph pattern Conv1x1 (-> LeakyRelu) -> DepthwiseConv3x3 ->
// Conv1x1 (-> Add) of the MBConv-style blocks, which the reference runs as
// three kernels with the expanded tensor (E channels, E = 2C in the block
// stack) and the depthwise result written to memory and read back
// (backends/driver_cubin/src/execution_plan.cpp:342-466: the pointwise GEMM
// path, then the depthwise kernel of :438-457, then the pointwise path again,
// each with the epilogue fusion of fusion_registry.cpp:711-800).  Here neither
// intermediate leaves the SM.  Per 16 x 8-pixel output tile (128 pixels, the
// MMA's M; row r of the tile = pixel (r % 16, r / 16)):
//
//   producer   TMA loads x over the tile's 18 x 10-pixel halo as one 3-D box
//              per 64 input channels, 128-byte swizzled: the box image is the
//              K-major SW128 A operand of the expand GEMM (halo row = pixel
//              (hr % 18, hr / 18)).  W1 / W2 panels stream through one ring.
//   MMA        per 64 expanded channels (a chunk): the expand GEMM over halo
//              rows 0..127 and 56..183 (two M = 128 blocks; rows 180..183 and
//              the repeated rows 56..127 of the second block are discarded)
//              into a double-buffered TMEM accumulator, then, once the
//              depthwise A panel of the chunk is ready, the projection GEMM
//              (K = 64) into the output accumulator.
//   expand     warps 2..9: the chunk's expand accumulators -> bias,
//              LeakyReLU, FP16, zero for halo pixels outside the image ->
//              the 180-row chunk of e in one of two shared-memory buffers
//   depthwise  warps 10..17: the depthwise conv of the previous chunk's 128
//              pixels x 64 channels into the SW128 A panel (4 channels x a
//              2 x 4 pixel block per thread), while the expand warps write
//              the next chunk; after the last chunk these warps run the
//              shared tile epilogue of the conv kernels for the output.
//
// The expand epilogue is the 1x1 conv kernel's (FP32 bias add, one rounding,
// LeakyReLU as fp16(fp32(h) * alpha) on negative halves), the depthwise and
// the projection are mlvc_dwconv_tc's, and the tensor core sums each row's K
// products in the same order whatever the tile shape, so the result is
// bit-identical to the three-kernel schedule.
//
// Roles (576 threads): warp 0 = TMA producer, warp 1 = TMEM owner (512
// columns: two expand accumulators of 2 x 64 columns, the output
// accumulator at column 256) + MMA issuer, warps 2..9 = expand epilogue,
// warps 10..17 = depthwise + output epilogue: the two CUDA-core stages use
// different units (TMEM loads and conversions; shared-memory loads and FMAs)
// and overlap chunk by chunk.  All waits are bounded (%globaltimer) and abort
// the CTA with an error bit in mlvc_b200_status; the warps hand buffers over
// through mbarriers (not named barriers), so an aborting thread never strands
// the others.
namespace mlvc_b200 {

struct MbShared {
    uint64_t x_full, x_empty;                        // x halo (all slices of a tile)
    uint64_t w_full[kMbWStages], w_empty[kMbWStages];  // W1 / W2 panel ring
    uint64_t acc1_full[2], acc1_empty[2];            // expand accumulators
    uint64_t a_full[2], a_empty[2];                  // depthwise A panels
    uint64_t acc2_full, acc2_empty;                  // output accumulator
    uint64_t e_full[2], e_empty[2];                  // e chunk buffers: written by the expand warps, read by the depthwise warps
    uint64_t stg_ready, stg_full;                    // output staging hand-over (see StageSync)
    uint64_t dw_full;                                // depthwise taps + bias landed
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
    alignas(16) float bias2[256];                    // projection bias, read as float2
    alignas(16) float bias1[kMbMaxExpand];           // expand bias, read as float2
};
static_assert(sizeof(MbShared) <= kMbHeaderBytes, "MbShared must fit the header reserved by the host");
static_assert(offsetof(MbShared, bias2) % 16 == 0 && offsetof(MbShared, bias1) % 16 == 0, "vector bias reads");
static_assert(kMbSliceBytes % 1024 == 0 && (kMbRow1 * 128) % 1024 == 0, "SW128 operands start on 1024-byte atoms");
static_assert(kMbRow1 + kBM == kMbHaloRows && kMbRow1 <= kBM, "the two expand M blocks cover halo rows 0..183");
static_assert(kDwHaloPx <= kMbHaloRows, "halo rows");

constexpr uint32_t kMbPanelBytes = kBM * 128;  // one 128-pixel x 64-channel FP16 panel
constexpr int kMbComputeThreads = 512;         // warps 2..17
constexpr int kMbThreads = kMbComputeThreads + 64;
constexpr int kMbExpandWarps = 8;              // warps 2..9
constexpr int kMbDwWarps = 8;                  // warps 10..17
constexpr int kMbDwThreads = kMbDwWarps * 32;
constexpr uint32_t kMbEBytes = kDwHaloPx * 128;  // one 64-channel FP16 chunk of e over the halo
static_assert(kMbThreads == kMbBlockThreads, "block size shared with the host");
static_assert(kMbDwThreads == kEpilogueThreads, "the depthwise warps run the shared output epilogue");

// One arrival per warp (these barriers count warps): the lanes' shared
// memory writes are ordered before lane 0's release by __syncwarp.
__device__ __forceinline__ void mb_warp_arrive(uint64_t* bar, int lane)
{
    __syncwarp();
    if (lane == 0)
        mbar_arrive(bar);
}
static_assert(kMbThreads == kMbBlockThreads, "block size shared with the host");
static_assert(kMbComputeThreads == 2 * kEpilogueThreads, "warps 2..9 also run the output epilogue");
constexpr uint32_t kMbAcc2Col = 256;           // output accumulator column in TMEM
constexpr uint32_t kMbTmemCols = 512;

// Weight panel j of a tile's sequence (the MMA issuer consumes them in this
// order): the expand GEMM runs two chunks ahead of the projection, so it
// never waits behind a projection slice whose depthwise panel is not ready:
// W1(0), W1(1), then W1(c), W2(c - 2) for c = 2 .. chunks - 1, then the last
// two W2 slices.  kind 0 = W1 (expand) chunk, 1 = W2 (projection) K slice.
__device__ __forceinline__ void mb_panel(int j, int nch, int& kind, int& c)
{
    const int lead = nch < 2 ? nch : 2;
    if (j < lead) {
        kind = 0;
        c = j;
        return;
    }
    j -= lead;
    const int steady = 2 * (nch - lead);
    if (j < steady) {
        kind = j & 1;
        c = (j & 1) ? j / 2 : lead + j / 2;
        return;
    }
    kind = 1;
    c = nch - lead + (j - steady);
}

// One thread, one halo row of one expand chunk: 16 accumulators (columns
// col0 .. col0 + 15 of the chunk) -> bias, the expand conv's operator, FP16,
// or +0 for a pixel outside the image -> 2 swizzled 16-byte chunks of row hr.
__device__ __forceinline__ void mb_expand_row(const MbConvTcParams& mp, const float* bias1, const uint32_t (&a)[16],
                                              int col0, int hr, bool inside, uint8_t* e_smem)
{
    uint32_t h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float2 b2 = *reinterpret_cast<const float2*>(&bias1[col0 + 2 * i]);
        h[i] = pack_h2(__uint_as_float(a[2 * i]) + b2.x, __uint_as_float(a[2 * i + 1]) + b2.y);
    }
    if (mp.epi1 == kEpiLeaky) {
        // negative halves become fp16(fp32(x) * alpha), as in the 1x1 conv epilogue
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float x0, x1;
            unpack_h2(h[i], x0, x1);
            const uint32_t m = pack_h2(x0 * mp.alpha1, x1 * mp.alpha1);
            const uint32_t neg = ((h[i] >> 15) & 0x00010001u) * 0xFFFFu;
            h[i] = (m & neg) | (h[i] & ~neg);
        }
    }
    const uint32_t keep = inside ? 0xFFFFFFFFu : 0u;  // the depthwise pads e with zeros
    uint8_t* row = e_smem + hr * 128;
    const int q0 = (col0 & 63) >> 3;
#pragma unroll
    for (int q = 0; q < 2; ++q)
        *reinterpret_cast<uint4*>(row + (((q0 + q) ^ (hr & 7)) << 4)) =
            make_uint4(h[4 * q] & keep, h[4 * q + 1] & keep, h[4 * q + 2] & keep, h[4 * q + 3] & keep);
}

extern "C" __global__ void __launch_bounds__(kMbThreads, 1) mlvc_mbconv_tc(const __grid_constant__ MbConvTcParams mp)
{
    const ConvTcParams& p = mp.c;
    extern __shared__ __align__(1024) uint8_t smem_dyn[];
    uint8_t* base = align_smem_1024(smem_dyn);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    MbShared* sh = reinterpret_cast<MbShared*>(base);

    const int kpx = mp.c_in / 64;       // 64-channel slices of x
    const int nch = mp.expand / 64;     // expand chunks
    const int nseq = 2 * nch;           // weight panels per tile
    const int panels = p.BN / 64;       // output panels
    uint8_t* x_smem = base + kMbHeaderBytes;
    uint8_t* e_smem = x_smem + static_cast<size_t>(kpx) * kMbSliceBytes;  // two e chunk buffers
    uint8_t* a_smem = e_smem + 2 * kMbEBytes;
    uint8_t* w_smem = a_smem + 2 * kMbPanelBytes;
    uint8_t* stage_smem = w_smem + kMbWStages * kMbWSlotBytes;  // 1024-aligned
    // depthwise taps [9][E] and bias [E], FP16, loaded once per CTA by TMA
    const uint8_t* dw_smem = stage_smem + static_cast<size_t>(panels) * kTcStagePanelBytes;

    if (threadIdx.x == 0) {
        if (p.trace)
            p.trace[blockIdx.x * kTracePoints + kTrEntry] = globaltimer_ns();
        mbar_init(&sh->x_full, 1);
        mbar_init(&sh->x_empty, 1);
        for (int s = 0; s < kMbWStages; ++s) {
            mbar_init(&sh->w_full[s], 1);
            mbar_init(&sh->w_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&sh->acc1_full[s], 1);
            mbar_init(&sh->acc1_empty[s], kMbExpandWarps);
            mbar_init(&sh->a_full[s], kMbDwWarps);
            mbar_init(&sh->a_empty[s], 1);
            mbar_init(&sh->e_full[s], kMbExpandWarps);
            mbar_init(&sh->e_empty[s], kMbDwWarps);
        }
        mbar_init(&sh->acc2_full, 1);
        mbar_init(&sh->acc2_empty, kEpilogueThreads);
        mbar_init(&sh->stg_ready, 1);
        mbar_init(&sh->stg_full, kEpilogueThreads);
        mbar_init(&sh->dw_full, 1);
        mbar_init(&sh->drain, 1);
        sh->abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && elect_one()) {
        tma_prefetch_desc(&mp.map_x);
        tma_prefetch_desc(&mp.map_w1);
        tma_prefetch_desc(&mp.map_dw);
        tma_prefetch_desc(&p.map_b);
        tma_prefetch_desc(&p.map_out);
        if (p.epilogue == kEpiResidual)
            tma_prefetch_desc(&p.map_res);
    }
    __syncthreads();
    if (threadIdx.x == 0)
        trace(p, kTrSetup);
    pdl_launch_dependents();

    const int first = blockIdx.x, step = gridDim.x, tiles = p.m_tiles;
    bool mma_thread = false;
    uint32_t issued = 0;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (elect_one()) {
            ArmedSlots w_armed, x_armed, dw_armed;
            int ws = 0;
            uint32_t wph = 0;
            const uint32_t w1_bytes = static_cast<uint32_t>(64 * mp.c_in * 2);
            const uint32_t w2_bytes = static_cast<uint32_t>(p.BN) * 128u;
            auto issue_w = [&](int j) -> bool {
                if (!mbar_wait(&sh->w_empty[ws], wph ^ 1u, &sh->abort_flag, kErrWaitProducer))
                    return false;
                uint8_t* dst = w_smem + static_cast<size_t>(ws) * kMbWSlotBytes;
                int kind, c;
                mb_panel(j, nch, kind, c);
                if (kind == 0) {
                    mbar_arrive_expect_tx(&sh->w_full[ws], w1_bytes);
                    for (int s = 0; s < kpx; ++s)
                        tma_load_2d(dst + s * 8192, &mp.map_w1, &sh->w_full[ws], s * 64, c * 64);
                } else {
                    mbar_arrive_expect_tx(&sh->w_full[ws], w2_bytes);
                    tma_load_2d(dst, &p.map_b, &sh->w_full[ws], c * 64, 0);
                }
                w_armed.arm(ws, wph);
                if (++ws == kMbWStages) {
                    ws = 0;
                    wph ^= 1u;
                }
                return true;
            };
            // The weights do not depend on the previous kernel.
            mbar_arrive_expect_tx(&sh->dw_full, static_cast<uint32_t>(10 * mp.expand * 2));
            tma_load_2d(const_cast<uint8_t*>(dw_smem), &mp.map_dw, &sh->dw_full, 0, 0);
            dw_armed.arm(0, 0);
            int w_issued = 0;  // panels issued, counted over the CTA's tiles
            if (first < tiles)
                for (; w_issued < min(nseq, kMbWStages); ++w_issued)
                    issue_w(w_issued);
            trace(p, kTrWeightsIssued);
            pdl_wait();  // x is written by the previous kernel
            trace(p, kTrDepReady);
            bool ok = true;
            int local = 0;
            for (int t = first; ok && t < tiles && !sh->abort_flag; t += step, ++local) {
                const int hx = (t % mp.tiles_x) * kDwTileW - 1, hy = (t / mp.tiles_x) * kDwTileH - 1;  // may be -1
                if (!mbar_wait(&sh->x_empty, (static_cast<uint32_t>(local) & 1u) ^ 1u, &sh->abort_flag,
                               kErrWaitProducer))
                    break;
                mbar_arrive_expect_tx(&sh->x_full, static_cast<uint32_t>(kpx * kDwHaloPx * 128));
                for (int s = 0; s < kpx; ++s)
                    tma_load_3d(x_smem + static_cast<size_t>(s) * kMbSliceBytes, &mp.map_x, &sh->x_full, s * 64, hx, hy);
                x_armed.arm(0, static_cast<uint32_t>(local) & 1u);
                for (; ok && w_issued < (local + 1) * nseq; ++w_issued)
                    ok = issue_w(w_issued % nseq);
            }
            if (sh->abort_flag) {
                drain_armed(&sh->x_full, x_armed, 1);
                drain_armed(sh->w_full, w_armed, kMbWStages);
                drain_armed(&sh->dw_full, dw_armed, 1);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------ TMEM owner + MMA issuer
        tmem_alloc(&sh->tmem_base, kMbTmemCols);
        tc_fence_before();
        asm volatile("bar.arrive 1, %0;" ::"n"(kMbComputeThreads + 32) : "memory");
        __syncwarp();
        tc_fence_after();
        if (elect_one()) {
            mma_thread = true;
            const uint32_t idesc1 = idesc_f16_f32(kBM, 64u), idesc2 = idesc_f16_f32(kBM, static_cast<uint32_t>(p.BN));
            const uint32_t x_addr = smem_u32(x_smem), a_addr = smem_u32(a_smem), w_addr = smem_u32(w_smem);
            int ws = 0, as = 0;
            uint32_t wph = 0, aph = 0, k1 = 0, local = 0;
            bool ok = true;
            for (int t = first; ok && t < tiles; t += step, ++local) {
                if (!mbar_wait(&sh->x_full, local & 1u, &sh->abort_flag, kErrWaitMma))
                    break;
                for (int j = 0; j < nseq; ++j) {
                    int kind, c;
                    mb_panel(j, nch, kind, c);
                    const uint32_t b_st = w_addr + static_cast<uint32_t>(ws) * kMbWSlotBytes;
                    if (kind == 0) {
                        // expand chunk c over both M blocks into acc1[k1 & 1]
                        const uint32_t buf = k1 & 1u;
                        if (!mbar_wait(&sh->acc1_empty[buf], ((k1 >> 1) & 1u) ^ 1u, &sh->abort_flag, kErrWaitMma) ||
                            !mbar_wait(&sh->w_full[ws], wph, &sh->abort_flag, kErrWaitMma)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        if (issued == 0)
                            trace(p, kTrFirstA);
                        if (local == 0 && c < 4)
                            trace(p, kTrMbExpandMma + c);
                        const uint32_t d = sh->tmem_base + buf * 128u;
#pragma unroll
                        for (int mb = 0; mb < 2; ++mb)
                            for (int s = 0; s < kpx; ++s)
#pragma unroll
                                for (int ks = 0; ks < 4; ++ks) {
                                    const uint32_t a = x_addr + static_cast<uint32_t>(s) * kMbSliceBytes +
                                                       static_cast<uint32_t>(mb * kMbRow1 * 128 + ks * 32);
                                    const uint32_t b = b_st + static_cast<uint32_t>(s * 8192 + ks * 32);
                                    umma_f16(d + static_cast<uint32_t>(mb * 64), smem_desc(a, 16, 1024, 2),
                                             smem_desc(b, 16, 1024, 2), idesc1, (s | ks) != 0);
                                    ++issued;
                                }
                        umma_commit(&sh->w_empty[ws]);
                        umma_commit(&sh->acc1_full[buf]);
                        if (c == nch - 1)
                            umma_commit(&sh->x_empty);  // the halo is free for the next tile
                        ++k1;
                    } else {
                        // projection K slice c from the depthwise A panel
                        if ((c == 0 && !mbar_wait(&sh->acc2_empty, (local & 1u) ^ 1u, &sh->abort_flag, kErrWaitMma)) ||
                            !mbar_wait(&sh->a_full[as], aph, &sh->abort_flag, kErrWaitMma) ||
                            !mbar_wait(&sh->w_full[ws], wph, &sh->abort_flag, kErrWaitMma)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        if (local == 0 && c < 4)
                            trace(p, kTrMbProjMma + c);
                        const uint32_t a_st = a_addr + static_cast<uint32_t>(as) * kMbPanelBytes;
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks) {
                            umma_f16(sh->tmem_base + kMbAcc2Col, smem_desc(a_st + ks * 32, 16, 1024, 2),
                                     smem_desc(b_st + ks * 32, 16, 1024, 2), idesc2, (c | ks) != 0);
                            ++issued;
                        }
                        umma_commit(&sh->a_empty[as]);
                        umma_commit(&sh->w_empty[ws]);
                        if (c == nch - 1)
                            umma_commit(&sh->acc2_full);
                        if (++as == 2) {
                            as = 0;
                            aph ^= 1u;
                        }
                    }
                    if (++ws == kMbWStages) {
                        ws = 0;
                        wph ^= 1u;
                    }
                }
            }
            trace(p, kTrLastCommit);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ expand epilogue / depthwise + output epilogue
        const int quadrant = warp & 3;
        const bool expand_role = warp < 2 + kMbExpandWarps;
        const int group = expand_role ? (warp - 2) / 4 : (warp - 2 - kMbExpandWarps) / 4;  // 0 or 1
        const int rt = (expand_role ? warp - 2 : warp - 2 - kMbExpandWarps) * 32 + lane;    // 0..255 in the role
        const bool leader = rt == 0;
        for (int i = (warp - 2) * 32 + lane; i < p.BN; i += kMbComputeThreads)
            sh->bias2[i] = (p.bias && i < p.N) ? __half2float(p.bias[i]) : 0.0f;
        for (int i = (warp - 2) * 32 + lane; i < mp.expand; i += kMbComputeThreads)
            sh->bias1[i] = mp.bias1 ? __half2float(mp.bias1[i]) : 0.0f;
        asm volatile("bar.sync 1, %0;" ::"n"(kMbComputeThreads + 32) : "memory");  // biases + TMEM address
        tc_fence_after();
        pdl_wait();  // residual reads and output writes follow the previous kernel
        const int W = mp.width, H = mp.height;
        bool ok = true;
        uint32_t kc = 0, it = 0;
        if (expand_role) {
            // this thread's expand rows: halo row r0 = its TMEM lane in block 0;
            // in block 1 lane L holds halo row kMbRow1 + L, new (>= 128, < 180)
            // only for lanes 72 .. 123, i.e. quadrants 2 and 3
            const int r0 = quadrant * 32 + lane, r1 = kMbRow1 + r0;
            const bool block1 = quadrant >= 2;  // warp-uniform
            const bool r1_new = r1 >= kBM && r1 < kDwHaloPx;
            const uint32_t lane_addr = static_cast<uint32_t>(quadrant * 32) << 16;
            for (int t = first; ok && t < tiles; t += step, ++it) {
                const int ox0 = (t % mp.tiles_x) * kDwTileW, oy0 = (t / mp.tiles_x) * kDwTileH;
                auto inside = [&](int hr) {
                    const int ix = ox0 - 1 + hr % (kDwTileW + 2), iy = oy0 - 1 + hr / (kDwTileW + 2);
                    return ix >= 0 && ix < W && iy >= 0 && iy < H;
                };
                const bool in0 = inside(r0), in1 = inside(r1);
                for (int c = 0; c < nch; ++c, ++kc) {
                    const uint32_t buf = kc & 1u, use = kc >> 1;
                    if (!mbar_wait(&sh->acc1_full[buf], use & 1u, &sh->abort_flag, kErrWaitEpilogue) ||
                        !mbar_wait(&sh->e_empty[buf], (use & 1u) ^ 1u, &sh->abort_flag, kErrWaitEpilogue)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (leader && it == 0 && c < 4)
                        trace(p, kTrMbChunk + 3 * c);
                    uint8_t* e_buf = e_smem + buf * kMbEBytes;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {  // 16 of the warpgroup's 32 columns at a time
                        const int col = group * 32 + h * 16;
                        const uint32_t acc = sh->tmem_base + lane_addr + buf * 128u + static_cast<uint32_t>(col);
                        uint32_t a0[16], a1[16];
                        tmem_ld16_nowait(acc, a0);
                        if (block1)
                            tmem_ld16_nowait(acc + 64u, a1);
                        tmem_wait_ld();
                        mb_expand_row(mp, sh->bias1, a0, c * 64 + col, r0, in0, e_buf);
                        if (block1 && r1_new)
                            mb_expand_row(mp, sh->bias1, a1, c * 64 + col, r1, in1, e_buf);
                    }
                    tc_fence_before();
                    mb_warp_arrive(&sh->acc1_empty[buf], lane);
                    mb_warp_arrive(&sh->e_full[buf], lane);
                    if (leader && it == 0 && c < 4)
                        trace(p, kTrMbChunk + 3 * c + 1);
                }
            }
        } else {
            // depthwise: 4 channels (cq) x a 2 x 4 pixel block (pb) per thread
            const int cq = rt & 15;
            const int pb = rt >> 4;                       // 0..15
            const int by = (pb >> 2) * 2, bx = (pb & 3) * 4;  // block: tile rows by, by + 1, columns bx .. bx + 3
            const int cq_chunk = cq >> 1, cq_half = (cq & 1) * 8;  // byte offset of the 4 channels in a row
            const StageSync ss{&sh->stg_ready, &sh->stg_full};
            ok = mbar_wait(&sh->dw_full, 0, &sh->abort_flag, kErrWaitEpilogue);
            int as = 0;
            uint32_t aph = 0;
            bool res_issued = false;  // the leader issued tile `it`'s residual load
            for (int t = first; ok && t < tiles; t += step, ++it) {
                TileCoord tc;
                tc.pixel0 = 0;
                tc.ox0 = (t % mp.tiles_x) * kDwTileW;
                tc.oy = (t / mp.tiles_x) * kDwTileH;
                if (leader)  // residual tile into the staging buffer while the block runs
                    stage_prepare(p, stage_smem, panels, 0, tc, true, p.epilogue == kEpiResidual, ss.ready);
                res_issued = p.epilogue == kEpiResidual;
                const int x0 = tc.ox0 + bx;
                for (int c = 0; c < nch; ++c, ++kc) {
                    const uint32_t buf = kc & 1u, use = kc >> 1;
                    if (!mbar_wait(&sh->e_full[buf], use & 1u, &sh->abort_flag, kErrWaitEpilogue) ||
                        !mbar_wait(&sh->a_empty[as], aph ^ 1u, &sh->abort_flag, kErrWaitEpilogue)) {
                        ok = false;
                        break;
                    }
                    const uint8_t* e_buf = e_smem + buf * kMbEBytes;
                    const int ch = c * 64 + cq * 4;
                    float acc[2][4][4];  // [row][column][channel]
                    {
                        float b4[4];
                        const uint2 bv = *reinterpret_cast<const uint2*>(dw_smem + (9 * mp.expand + ch) * 2);
                        unpack_h2(bv.x, b4[0], b4[1]);
                        unpack_h2(bv.y, b4[2], b4[3]);
#pragma unroll
                        for (int j = 0; j < 2; ++j)
#pragma unroll
                            for (int i = 0; i < 4; ++i)
#pragma unroll
                                for (int k = 0; k < 4; ++k)
                                    acc[j][i][k] = b4[k];
                    }
                    uint32_t wv[9][2];
#pragma unroll
                    for (int tap = 0; tap < 9; ++tap) {
                        const uint2 q = *reinterpret_cast<const uint2*>(dw_smem + (tap * mp.expand + ch) * 2);
                        wv[tap][0] = q.x;
                        wv[tap][1] = q.y;
                    }
                    // e columns x0 - 1 .. x0 + 4 over halo rows by .. by + 3; output
                    // pixel (j, i) takes column cc with kx = cc - i and halo row j + ky
#pragma unroll
                    for (int cc = 0; cc < 6; ++cc) {
                        const int ix = x0 - 1 + cc;
                        if (ix < 0 || ix >= W)
                            continue;  // outside the image: the tap is skipped (no padding term)
                        uint32_t xv[4][2];
#pragma unroll
                        for (int rr = 0; rr < 4; ++rr) {
                            const int hr = (by + rr) * (kDwTileW + 2) + bx + cc;
                            const uint2 v =
                                *reinterpret_cast<const uint2*>(e_buf + hr * 128 + ((cq_chunk ^ (hr & 7)) << 4) + cq_half);
                            xv[rr][0] = v.x;
                            xv[rr][1] = v.y;
                        }
#pragma unroll
                        for (int j = 0; j < 2; ++j)
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const int kx = cc - i;
                                if (kx < 0 || kx > 2)
                                    continue;
#pragma unroll
                                for (int ky = 0; ky < 3; ++ky)
#pragma unroll
                                    for (int k = 0; k < 2; ++k)
                                        fma_h2(acc[j][i][2 * k], acc[j][i][2 * k + 1], xv[j + ky][k], wv[ky * 3 + kx][k]);
                            }
                    }
                    mb_warp_arrive(&sh->e_empty[buf], lane);  // e chunk read
                    // rounded depthwise output -> A panel row r (tile pixel (bx + i, by + j)), 128-byte swizzle
                    uint8_t* apanel = a_smem + static_cast<size_t>(as) * kMbPanelBytes;
#pragma unroll
                    for (int j = 0; j < 2; ++j)
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int r = (by + j) * kDwTileW + bx + i;
                            *reinterpret_cast<uint2*>(apanel + r * 128 + ((cq_chunk ^ (r & 7)) << 4) + cq_half) =
                                make_uint2(pack_h2(acc[j][i][0], acc[j][i][1]), pack_h2(acc[j][i][2], acc[j][i][3]));
                        }
                    fence_proxy_async_smem();  // the tensor core reads the panel through the async proxy
                    mb_warp_arrive(&sh->a_full[as], lane);
                    if (leader && it == 0) {
                        if (c == 0)
                            trace(p, kTrDwFirstSlice);
                        if (c < 4)
                            trace(p, kTrMbChunk + 3 * c + 2);
                    }
                    if (++as == 2) {
                        as = 0;
                        aph ^= 1u;
                    }
                }
                if (!ok)
                    break;
                if (!epilogue_tile(p, sh->bias2, sh->tmem_base + kMbAcc2Col, &sh->acc2_full, it & 1u, &sh->acc2_empty,
                                   ss, it, stage_smem, nullptr, panels, 0, tc, true, quadrant, group, lane, leader,
                                   &sh->abort_flag)) {
                    ok = false;
                    break;
                }
                if (leader && it == 0)
                    trace(p, kTrFirstAcc);
            }
            if (leader) {
                // An aborted tile's residual load may still be in flight: wait
                // (bounded) for its barrier phase before shared memory retires.
                if (!ok && res_issued) {
                    volatile int never = 0;
                    mbar_wait(ss.ready, it & 1u, &never, kErrWaitEpilogue);
                }
                bulk_wait_all();
                trace(p, kTrEpilogueDone);
            }
        }
    }

    if (mma_thread && sh->abort_flag && issued) {
        umma_commit(&sh->drain);
        volatile int never = 0;
        mbar_wait(&sh->drain, 0, &never, kErrWaitMma);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(sh->tmem_base, kMbTmemCols);
    }
    if (threadIdx.x == 0)
        trace(p, kTrExit);
}

}  // namespace mlvc_b200
