// Fused depthwise 3x3 + 1x1 conv for sm_100a (CUDA cores + tcgen05 + TMA):
//
//     d   = fp16(dw3x3(x) + b_dw)           stride 1, pad 1, FP32 FMA from the bias
//     out = epilogue(fp16(d W^T + b))       bias / LeakyReLU / + residual
//
// This is the graph pattern DepthwiseConv3x3 -> Conv1x1 (-> Add | LeakyRelu)
// of the MBConv-style blocks, which the reference runs as a depthwise kernel
// writing the C-channel tensor to memory and a GEMM reading it back
// (backends/driver_cubin/src/execution_plan.cpp:438-457, then the pointwise
// path of :134-269 with the epilogue fusion of fusion_registry.cpp:711-800).
// Here the depthwise result never leaves the SM: per 16 x 8-pixel tile
// (128 pixels, the MMA's M; row r of the tile = pixel (r % 16, r / 16)) and
// per 64-channel slice,
//
//   producer   TMA loads the slice's 18 x 10-pixel halo as one 3-D box (the
//              TMA zero fill outside the image is the padding of the top and
//              bottom rows; columns outside the image are skipped below)
//   CUDA cores 256 threads compute the depthwise conv of the 128 pixels x 64
//              channels (8 channels x 4 horizontally adjacent pixels each,
//              every input column loaded once) and write it, rounded to FP16,
//              as the K-major 128-byte-swizzled A panel of the GEMM
//   MMA        one thread issues 4 tcgen05.mma (K = 16 each) of the slice into
//              the TMEM accumulator, the weight panel streamed by TMA
//
// and the shared tile epilogue of the conv kernels stores the output.  The
// depthwise arithmetic (FP32 accumulation from the bias, taps in kx-major /
// ky-minor order, columns outside the image skipped, one rounding) is the
// stand-alone depthwise kernel's, so the result is bit-identical to the
// unfused pair.
//
// Roles (448 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA
// issuer, warps 2..9 = depthwise compute, warps 10..13 = output epilogue (one
// per TMEM lane quadrant).  The accumulator is double-buffered, so tile t's
// epilogue (TMEM -> bias, fused operator -> staging -> TMA store) overlaps
// tile t + 1's depthwise slices.  All waits are bounded (%globaltimer) and
// abort the CTA with an error bit in mlvc_b200_status.
namespace mlvc_b200 {

struct DwShared {
    uint64_t h_full[2], h_empty[2];  // halo slices
    uint64_t a_full[2], a_empty[2];  // depthwise A panels
    uint64_t w_full[2], w_empty[2];  // 1x1 weight panels
    uint64_t acc_full[2], acc_empty[2];
    uint64_t stg_ready, stg_full;    // output staging hand-over (see StageSync)
    uint64_t dw_full;                // depthwise taps + bias landed
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
    alignas(16) float bias[256];     // 1x1 conv bias, read as float2
};
static_assert(sizeof(DwShared) <= kDwHeaderBytes, "DwShared must fit the header reserved by the host");
static_assert(offsetof(DwShared, bias) % 16 == 0, "vector bias reads");

constexpr uint32_t kDwPanelBytes = kBM * 128;  // one 128-pixel x 64-channel FP16 panel

extern "C" __global__ void __launch_bounds__(kDwThreads, 1) mlvc_dwconv_tc(const __grid_constant__ DwConvTcParams dp)
{
    const ConvTcParams& p = dp.c;
    extern __shared__ __align__(1024) uint8_t smem_dyn[];
    uint8_t* base = align_smem_1024(smem_dyn);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    DwShared* sh = reinterpret_cast<DwShared*>(base);

    const int kpan = p.K / 64;  // 64-channel slices per tile
    const uint32_t w_bytes = static_cast<uint32_t>(p.BN) * 128u;
    const uint32_t halo_stride = kDwHaloBytes;
    uint8_t* a_smem = base + kDwHeaderBytes;
    uint8_t* w_smem = a_smem + static_cast<size_t>(p.a_stages) * kDwPanelBytes;
    uint8_t* h_smem = w_smem + static_cast<size_t>(p.b_stages) * w_bytes;
    uint8_t* stage_smem = h_smem + static_cast<size_t>(dp.h_stages) * halo_stride;  // 1024-aligned
    // depthwise taps and bias, FP16, loaded once per CTA by TMA in groups of
    // tg = dw_tap_group(C) channels (a TMA box dimension is at most 256; the
    // groups tile C exactly): group g holds rows [10][tg] (rows 0..8: tap
    // ky * 3 + kx, row 9: bias) of channels g * tg .. g * tg + tg - 1
    const uint8_t* dw_smem = stage_smem + static_cast<size_t>(p.BN / 64) * kTcStagePanelBytes;
    const int tg = dw_tap_group(p.K);

    if (threadIdx.x == 0) {
        if (p.trace)
            p.trace[blockIdx.x * kTracePoints + kTrEntry] = globaltimer_ns();
        for (int s = 0; s < 2; ++s) {
            mbar_init(&sh->h_full[s], 1);
            mbar_init(&sh->h_empty[s], kDwComputeThreads);
            mbar_init(&sh->a_full[s], kDwComputeThreads);
            mbar_init(&sh->a_empty[s], 1);
            mbar_init(&sh->w_full[s], 1);
            mbar_init(&sh->w_empty[s], 1);
            mbar_init(&sh->acc_full[s], 1);
            mbar_init(&sh->acc_empty[s], kDwEpilogueThreads);
        }
        mbar_init(&sh->stg_ready, 1);
        mbar_init(&sh->stg_full, kDwEpilogueThreads);
        mbar_init(&sh->dw_full, 1);
        mbar_init(&sh->drain, 1);
        sh->abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && elect_one()) {
        tma_prefetch_desc(&dp.map_halo);
        tma_prefetch_desc(&dp.map_dw);
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
            ArmedSlots h_armed, w_armed;
            int hs = 0, ws = 0;
            uint32_t hph = 0, wph = 0;
            // weight panel kp of the 1x1 conv (the same sequence for every tile)
            auto issue_w = [&](int kp) -> bool {
                if (!mbar_wait(&sh->w_empty[ws], wph ^ 1u, &sh->abort_flag, kErrWaitProducer))
                    return false;
                mbar_arrive_expect_tx(&sh->w_full[ws], w_bytes);
                tma_load_2d(w_smem + static_cast<size_t>(ws) * w_bytes, &p.map_b, &sh->w_full[ws], kp * 64, 0);
                w_armed.arm(ws, wph);
                if (++ws == p.b_stages) {
                    ws = 0;
                    wph ^= 1u;
                }
                return true;
            };
            // The weights do not depend on the previous kernel.
            ArmedSlots dw_armed;
            mbar_arrive_expect_tx(&sh->dw_full, static_cast<uint32_t>(10 * p.K * 2));
            for (int g = 0; g * tg < p.K; ++g)
                tma_load_2d(const_cast<uint8_t*>(dw_smem) + static_cast<size_t>(g) * 10 * tg * 2, &dp.map_dw,
                            &sh->dw_full, g * tg, 0);
            dw_armed.arm(0, 0);
            int w_issued = 0;
            if (first < tiles)
                for (; w_issued < min(kpan, p.b_stages); ++w_issued)
                    issue_w(w_issued);
            trace(p, kTrWeightsIssued);
            pdl_wait();  // x is written by the previous kernel
            trace(p, kTrDepReady);
            int local = 0;
            bool ok = true;
            for (int t = first; ok && t < tiles && !sh->abort_flag; t += step, ++local) {
                const int hx = (t % dp.tiles_x) * kDwTileW - 1, hy = (t / dp.tiles_x) * kDwTileH - 1;  // may be -1
                for (int kp = 0; kp < kpan; ++kp) {
                    if (!mbar_wait(&sh->h_empty[hs], hph ^ 1u, &sh->abort_flag, kErrWaitProducer)) {
                        ok = false;
                        break;
                    }
                    uint8_t* dst = h_smem + static_cast<size_t>(hs) * halo_stride;
                    mbar_arrive_expect_tx(&sh->h_full[hs], static_cast<uint32_t>(kDwHaloPx) * 128u);
                    tma_load_3d(dst, &dp.map_halo, &sh->h_full[hs], kp * 64, hx, hy);
                    h_armed.arm(hs, hph);
                    if (++hs == dp.h_stages) {
                        hs = 0;
                        hph ^= 1u;
                    }
                    // keep the weight ring at least up to this slice
                    const int w_target = local * kpan + kp + 1;
                    for (; ok && w_issued < w_target; ++w_issued)
                        ok = issue_w(w_issued % kpan);
                }
            }
            if (sh->abort_flag) {
                drain_armed(sh->h_full, h_armed, dp.h_stages);
                drain_armed(sh->w_full, w_armed, p.b_stages);
                drain_armed(&sh->dw_full, dw_armed, 1);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------ TMEM owner + MMA issuer
        // accumulators (two buffers of BN columns), published to the epilogue
        // warps through named barrier 1 (128 epilogue threads + this warp)
        tmem_alloc(&sh->tmem_base, tmem_cols_for(p.BN));
        tc_fence_before();
        asm volatile("bar.arrive 1, %0;" ::"n"(kDwEpilogueThreads + 32) : "memory");
        __syncwarp();
        tc_fence_after();
        if (elect_one()) {
            mma_thread = true;
            const uint32_t idesc = idesc_f16_f32(kBM, static_cast<uint32_t>(p.BN));
            const uint32_t a_addr = smem_u32(a_smem), w_addr = smem_u32(w_smem);
            int as = 0, ws = 0;
            uint32_t aph = 0, wph = 0, acc = 0, acc_phase = 0;
            bool ok = true;
            for (int t = first; ok && t < tiles; t += step) {
                if (!mbar_wait(&sh->acc_empty[acc], acc_phase ^ 1u, &sh->abort_flag, kErrWaitMma))
                    break;
                tc_fence_after();
                const uint32_t d = sh->tmem_base + acc * static_cast<uint32_t>(p.BN);
                for (int kp = 0; kp < kpan; ++kp) {
                    if (!mbar_wait(&sh->a_full[as], aph, &sh->abort_flag, kErrWaitMma) ||
                        !mbar_wait(&sh->w_full[ws], wph, &sh->abort_flag, kErrWaitMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (issued == 0)
                        trace(p, kTrFirstA);
                    if (t == first && kp < 8)
                        trace(p, kTrDwMma + kp);
                    const uint32_t a_st = a_addr + static_cast<uint32_t>(as) * kDwPanelBytes;
                    const uint32_t b_st = w_addr + static_cast<uint32_t>(ws) * w_bytes;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        umma_f16(d, smem_desc(a_st + ks * 32, 16, 1024, 2), smem_desc(b_st + ks * 32, 16, 1024, 2), idesc,
                                 (kp | ks) != 0);
                        ++issued;
                    }
                    umma_commit(&sh->a_empty[as]);
                    umma_commit(&sh->w_empty[ws]);
                    if (++as == p.a_stages) {
                        as = 0;
                        aph ^= 1u;
                    }
                    if (++ws == p.b_stages) {
                        ws = 0;
                        wph ^= 1u;
                    }
                }
                if (!ok)
                    break;
                umma_commit(&sh->acc_full[acc]);
                acc ^= 1u;
                acc_phase ^= (acc == 0) ? 1u : 0u;
            }
            trace(p, kTrLastCommit);
        }
        __syncwarp();
    } else if (warp < 2 + kDwComputeThreads / 32) {
        // ------------------------------------------------ depthwise warps
        const int et_id = (warp - 2) * 32 + lane;
        const bool leader = et_id == 0;
        const int cq = et_id & 7;     // 8-channel chunk of the slice
        const int pg = et_id >> 3;    // pixels 4 pg .. 4 pg + 3 of the tile
        const int W = dp.width;
        bool ok = mbar_wait(&sh->dw_full, 0, &sh->abort_flag, kErrWaitEpilogue);
        int hs = 0, as = 0;
        uint32_t hph = 0, aph = 0, it = 0;
        for (int t = first; ok && t < tiles; t += step, ++it) {
            const int ox0 = (t % dp.tiles_x) * kDwTileW;
            const int ty = pg >> 2, tx = (pg & 3) * 4;  // the thread's 4 pixels: tile row ty, columns tx .. tx + 3
            const int x0 = ox0 + tx;
            const int h0 = (ty + 1) * (kDwTileW + 2) + tx + 1;  // halo pixel of the first one
            for (int kp = 0; kp < kpan; ++kp) {
                if (!mbar_wait(&sh->h_full[hs], hph, &sh->abort_flag, kErrWaitEpilogue) ||
                    !mbar_wait(&sh->a_empty[as], aph ^ 1u, &sh->abort_flag, kErrWaitEpilogue)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int ch = kp * 64 + cq * 8;
                // channel ch in the taps' group layout
                const uint8_t* taps = dw_smem + (static_cast<size_t>(ch / tg) * 10 * tg + ch % tg) * 2;
                float acc4[4][8];
                {
                    float b8[8];
                    const uint4 bv = *reinterpret_cast<const uint4*>(taps + 9 * tg * 2);
                    const uint32_t* bw = reinterpret_cast<const uint32_t*>(&bv);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        unpack_h2(bw[k], b8[2 * k], b8[2 * k + 1]);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
#pragma unroll
                        for (int k = 0; k < 8; ++k)
                            acc4[i][k] = b8[k];
                }
                // taps as packed FP16 pairs: the mixed-precision FMA needs no conversion
                uint32_t wv[9][4];
#pragma unroll
                for (int tap = 0; tap < 9; ++tap) {
                    const uint4 q = *reinterpret_cast<const uint4*>(taps + tap * tg * 2);
                    wv[tap][0] = q.x;
                    wv[tap][1] = q.y;
                    wv[tap][2] = q.z;
                    wv[tap][3] = q.w;
                }
                const uint8_t* halo = h_smem + static_cast<size_t>(hs) * halo_stride + cq * 16;
                // input columns x0 - 1 .. x0 + 4; output pixel i takes column cc with kx = cc - i
#pragma unroll
                for (int cc = 0; cc < 6; ++cc) {
                    const int ix = x0 - 1 + cc;
                    if (ix < 0 || ix >= W)
                        continue;  // outside the image: the tap is skipped (no padding term)
                    uint32_t xv[3][4];
#pragma unroll
                    for (int ky = 0; ky < 3; ++ky) {
                        const uint4 v =
                            *reinterpret_cast<const uint4*>(halo + static_cast<size_t>(h0 + (ky - 1) * (kDwTileW + 2) + cc - 1) * 128);
                        xv[ky][0] = v.x;
                        xv[ky][1] = v.y;
                        xv[ky][2] = v.z;
                        xv[ky][3] = v.w;
                    }
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int kx = cc - i;
                        if (kx < 0 || kx > 2)
                            continue;
#pragma unroll
                        for (int ky = 0; ky < 3; ++ky)
#pragma unroll
                            for (int k = 0; k < 4; ++k)
                                fma_h2(acc4[i][2 * k], acc4[i][2 * k + 1], xv[ky][k], wv[ky * 3 + kx][k]);
                    }
                }
                mbar_arrive(&sh->h_empty[hs]);  // halo slice read
                // rounded depthwise output -> A panel row (4 pg + i), 128-byte swizzle
                uint8_t* apanel = a_smem + static_cast<size_t>(as) * kDwPanelBytes;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int r = 4 * pg + i;
                    uint4 ov;
                    uint32_t* o = reinterpret_cast<uint32_t*>(&ov);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        o[k] = pack_h2(acc4[i][2 * k], acc4[i][2 * k + 1]);
                    *reinterpret_cast<uint4*>(apanel + r * 128 + ((cq ^ (r & 7)) << 4)) = ov;
                }
                fence_proxy_async_smem();  // the tensor core reads the panel through the async proxy
                mbar_arrive(&sh->a_full[as]);
                if (leader && it == 0 && kp == 0)
                    trace(p, kTrDwFirstSlice);
                if (leader && it == 0 && kp < 8)
                    trace(p, kTrDwSlice + kp);
                if (leader && it == 1 && kp == 0)
                    trace(p, kTrDwTile1);
                if (++hs == dp.h_stages) {
                    hs = 0;
                    hph ^= 1u;
                }
                if (++as == p.a_stages) {
                    as = 0;
                    aph ^= 1u;
                }
            }
        }
    } else {
        // ------------------------------------------------ output epilogue warps
        // (one per TMEM lane quadrant): tile t's accumulator is stored while
        // the depthwise warps compute tile t + 1
        const int quadrant = warp & 3;
        const int e_id = (warp - 2 - kDwComputeThreads / 32) * 32 + lane;
        const bool leader = e_id == 0;
        for (int i = e_id; i < p.BN; i += kDwEpilogueThreads)
            sh->bias[i] = (p.bias && i < p.N) ? __half2float(p.bias[i]) : 0.0f;
        asm volatile("bar.sync 1, %0;" ::"n"(kDwEpilogueThreads + 32) : "memory");  // bias + TMEM address
        tc_fence_after();
        pdl_wait();  // residual reads and output writes follow the previous kernel
        const StageSync ss{&sh->stg_ready, &sh->stg_full};
        const int panels = p.BN / 64;
        uint32_t acc = 0, acc_phase = 0, it = 0;
        bool ok = true;
        bool res_issued = false;  // the leader issued tile `it`'s residual load
        for (int t = first; t < tiles; t += step, ++it) {
            TileCoord tc;
            tc.pixel0 = 0;
            tc.ox0 = (t % dp.tiles_x) * kDwTileW;
            tc.oy = (t / dp.tiles_x) * kDwTileH;
            // the previous tile's store must have read the staging buffer; the
            // residual tile then lands in it while the depthwise runs
            if (leader) {
                stage_prepare(p, stage_smem, panels, 0, tc, true, p.epilogue == kEpiResidual, ss.ready);
                res_issued = p.epilogue == kEpiResidual;
            }
            if (!epilogue_tile(p, sh->bias, sh->tmem_base + acc * p.BN, &sh->acc_full[acc], acc_phase, &sh->acc_empty[acc],
                               ss, it, stage_smem, nullptr, panels, 0, tc, true, quadrant, 0, lane, leader,
                               &sh->abort_flag, 1)) {
                ok = false;
                break;
            }
            res_issued = false;
            if (leader && it == 0)
                trace(p, kTrFirstAcc);
            acc ^= 1u;
            acc_phase ^= (acc == 0) ? 1u : 0u;
        }
        if (leader) {
            // An aborted tile's residual load may still be in flight: wait
            // (bounded) for its barrier phase before shared memory retires; a
            // phase that already completed returns at once.
            if (!ok && res_issued) {
                volatile int never = 0;
                mbar_wait(ss.ready, it & 1u, &never, kErrWaitEpilogue);
            }
            bulk_wait_all();
            trace(p, kTrEpilogueDone);
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
        tmem_dealloc(sh->tmem_base, tmem_cols_for(p.BN));
    }
    if (threadIdx.x == 0)
        trace(p, kTrExit);
}

}  // namespace mlvc_b200
