// Fused feed-forward block for sm_100a (tcgen05 + TMEM + TMA):
//
//     hidden = ReGLU(X W1^T + b1)            gate = first half, linear = second
//     out    = epilogue(hidden W2^T + b2)    bias / LeakyReLU / + residual
//
// This is the graph pattern Conv1x1(C -> 2H) -> Slice -> Slice -> Clip -> Mul
// -> Conv1x1(H -> C_out) (-> Add | LeakyRelu) that the reference runs as a
// ReGLU GEMM followed by a second GEMM with the H-channel tensor written to
// and re-read from memory (backends/driver_cubin/src/fusion_registry.cpp:
// 893-1036 then 711-800).  Here the hidden tensor never leaves the SM: per
// 128-pixel tile the hidden channels are produced 64 at a time,
//
//   GEMM1 chunk j   X[128 x C] . W1[j]^T[C x 128] -> TMEM acc1 (64 gate + 64 linear columns)
//   ReGLU epilogue  acc1 -> bias, FP16 rounding, clip, product, rounding -> shared memory,
//                   written in the 128-byte-swizzled K-major layout the tensor core reads
//   GEMM2 chunk j   hidden_j[128 x 64] . W2[:, j]^T -> TMEM acc2 (accumulated over chunks)
//
// and the output epilogue (shared with the conv kernels) runs once per tile.
// Rounding is the graph's operator-by-operator rounding (reference semantics:
// backends/cpu/src/kernels_scalar.cpp:180-192 and 304-322), so the result
// equals the unfused three-kernel schedule.
//
// Roles (320 threads): warp 0 = TMA producer (X tiles, then one weight ring
// in the exact order the MMAs consume it), warp 1 = TMEM owner (512 columns:
// two acc1 buffers of 128, acc2 buffers after them) + MMA issuer, warps 2..9 =
// ReGLU and output epilogues.  The MMA issuer runs GEMM1 two chunks ahead of
// GEMM2, so the tensor core works while the epilogue converts a chunk.  All waits are bounded (%globaltimer) and abort the CTA with an error
// bit in mlvc_b200_status.
namespace mlvc_b200 {

struct FfnShared {
    uint64_t x_full[2], x_empty[2];
    uint64_t w_full[kFfnMaxWStages], w_empty[kFfnMaxWStages];
    uint64_t acc1_full[2], acc1_empty[2];
    uint64_t hid_full[2], hid_empty[2];
    uint64_t acc2_full[2], acc2_empty[2];
    uint64_t stg_ready, stg_full;  // hidden/staging panel hand-over (see StageSync)
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
    alignas(16) float bias2[256];             // read as float2
    alignas(16) float bias1[2 * kFfnMaxHidden];  // read as float4
};
static_assert(sizeof(FfnShared) <= kFfnHeaderBytes, "FfnShared must fit the header reserved by the host");
static_assert(offsetof(FfnShared, bias1) % 16 == 0 && offsetof(FfnShared, bias2) % 16 == 0, "vector bias reads");

constexpr uint32_t kFfnTmemCols = 512;
constexpr uint32_t kFfnPanelBytes = kBM * 128;  // one 128-row x 64-channel FP16 panel

// GEMM2 of chunk j is issued after GEMM1 of chunk j + kFfnLag: GEMM1 of the
// next chunks then never queues behind a GEMM2 that waits for the epilogue,
// so the epilogue finds every acc1 chunk complete when it gets to it.
constexpr int kFfnLag = 2;

// Position idx (0 <= idx < per_tile) of the per-tile weight sequence, which is
// the MMA issue order: for j = 0 .. nch + kFfnLag - 1, the W1 panels of chunk
// j (j < nch), then the W2 panel of chunk j - kFfnLag (j >= kFfnLag).
__device__ __forceinline__ void ffn_weight_at(int idx, int kpan, int nch, int& chunk, int& kp, bool& w2)
{
    chunk = kp = 0;
    w2 = false;
    for (int j = 0; j < nch + kFfnLag; ++j) {
        if (j < nch) {
            if (idx < kpan) {
                chunk = j;
                kp = idx;
                return;
            }
            idx -= kpan;
        }
        if (j >= kFfnLag) {
            if (idx == 0) {
                chunk = j - kFfnLag;
                w2 = true;
                return;
            }
            idx -= 1;
        }
    }
}

extern "C" __global__ void __launch_bounds__(kThreads, 1) mlvc_ffn_tc(const __grid_constant__ FfnTcParams fp)
{
    const ConvTcParams& p = fp.c;
    extern __shared__ __align__(1024) uint8_t smem_dyn[];
    uint8_t* base = align_smem_1024(smem_dyn);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    FfnShared* sh = reinterpret_cast<FfnShared*>(base);

    const int kpan = p.K / 64;               // X panels per tile (and W1 panels per chunk)
    const int nch = fp.hidden / kFfnChunk;   // hidden chunks
    const int per_tile = nch * kpan + nch;   // weight panels per tile
    const uint32_t x_tile_bytes = static_cast<uint32_t>(kpan) * kFfnPanelBytes;
    const uint32_t slot_bytes = static_cast<uint32_t>(fp.w_slot_bytes);
    const uint32_t w2_bytes = static_cast<uint32_t>(p.BN) * 128u;
    const int acc2_bufs = p.BN <= 128 ? 2 : 1;
    uint8_t* x_smem = base + kFfnHeaderBytes;
    uint8_t* hid_smem = x_smem + static_cast<size_t>(p.a_stages) * x_tile_bytes;
    uint8_t* w_smem = hid_smem + 2 * kFfnPanelBytes;
    // The output epilogue stages the output tile in the hidden panels: they
    // are free once the tile's last GEMM2 completed (acc2 full) and go back to
    // the next tile's ReGLU epilogue once the TMA stores have read them.  The
    // residual (when the graph adds the FFN input) is read from the X tile,
    // which therefore stays resident until the output epilogue is done.
    uint8_t* stage_smem = hid_smem;

    if (threadIdx.x == 0) {
        if (p.trace)
            p.trace[blockIdx.x * kTracePoints + kTrEntry] = globaltimer_ns();
        for (int s = 0; s < 2; ++s) {
            mbar_init(&sh->x_full[s], 1);
            mbar_init(&sh->x_empty[s], 1 + kEpilogueThreads);  // last GEMM1 + the output epilogue's residual reads
            mbar_init(&sh->acc1_full[s], 1);
            mbar_init(&sh->acc1_empty[s], kEpilogueThreads);
            mbar_init(&sh->hid_full[s], kEpilogueThreads);
            mbar_init(&sh->hid_empty[s], 1);
            mbar_init(&sh->acc2_full[s], 1);
            mbar_init(&sh->acc2_empty[s], kEpilogueThreads);
        }
        for (int s = 0; s < kFfnMaxWStages; ++s) {
            mbar_init(&sh->w_full[s], 1);
            mbar_init(&sh->w_empty[s], 1);
        }
        mbar_init(&sh->stg_ready, 1);
        mbar_init(&sh->stg_full, kEpilogueThreads);
        mbar_init(&sh->drain, 1);
        sh->abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && elect_one()) {
        tma_prefetch_desc(&p.map_a0);
        tma_prefetch_desc(&p.map_b);
        tma_prefetch_desc(&fp.map_w2);
        tma_prefetch_desc(&p.map_out);
    }
    __syncthreads();
    if (threadIdx.x == 0)
        trace(p, kTrSetup);
    pdl_launch_dependents();

    const int first = blockIdx.x, step = gridDim.x, tiles = p.m_tiles;
    bool mma_thread = false;
    uint32_t issued = 0;

    if (warp == 0) {
        if (elect_one()) {
            ArmedSlots x_armed, w_armed;
            int ws = 0, xs = 0;
            uint32_t wph = 0, xph = 0;
            auto issue_w = [&](int idx) -> bool {
                if (!mbar_wait(&sh->w_empty[ws], wph ^ 1u, &sh->abort_flag, kErrWaitProducer))
                    return false;
                int chunk, kp;
                bool w2;
                ffn_weight_at(idx, kpan, nch, chunk, kp, w2);
                uint8_t* dst = w_smem + static_cast<size_t>(ws) * slot_bytes;
                if (!w2) {
                    mbar_arrive_expect_tx(&sh->w_full[ws], kFfnPanelBytes);
                    tma_load_2d(dst, &p.map_b, &sh->w_full[ws], kp * 64, chunk * 128);
                } else {
                    mbar_arrive_expect_tx(&sh->w_full[ws], w2_bytes);
                    tma_load_2d(dst, &fp.map_w2, &sh->w_full[ws], chunk * 64, 0);
                }
                w_armed.arm(ws, wph);
                if (++ws == p.b_stages) {
                    ws = 0;
                    wph ^= 1u;
                }
                return true;
            };
            // The weights do not depend on the previous kernel: the first GEMM's
            // panels go out before waiting for it, X right after the wait, and
            // the rest of the ring behind X (every TMA instruction occupies the
            // SM's copy engine for tens of nanoseconds, so X must not queue
            // behind the whole ring).
            int widx = 0;
            if (first < tiles)
                for (; widx < min(kpan, p.b_stages); ++widx)
                    issue_w(widx);
            trace(p, kTrWeightsIssued);
            pdl_wait();  // X is written by the previous kernel
            trace(p, kTrDepReady);
            int local = 0;
            for (int t = first; t < tiles && !sh->abort_flag; t += step, ++local) {
                if (!mbar_wait(&sh->x_empty[xs], xph ^ 1u, &sh->abort_flag, kErrWaitProducer))
                    break;
                uint8_t* xdst = x_smem + static_cast<size_t>(xs) * x_tile_bytes;
                mbar_arrive_expect_tx(&sh->x_full[xs], x_tile_bytes);
                for (int kp = 0; kp < kpan; ++kp)
                    tma_load_2d(xdst + kp * kFfnPanelBytes, &p.map_a0, &sh->x_full[xs], kp * 64, t * kBM);
                x_armed.arm(xs, xph);
                if (++xs == p.a_stages) {
                    xs = 0;
                    xph ^= 1u;
                }
                if (local == 0)
                    trace(p, kTrFfnXIssued);
                const int tile_end = (local + 1) * per_tile;
                for (; widx < tile_end; ++widx)
                    if (!issue_w(widx % per_tile))
                        break;
            }
            if (sh->abort_flag) {
                drain_armed(sh->x_full, x_armed, p.a_stages);
                drain_armed(sh->w_full, w_armed, p.b_stages);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        tmem_alloc(&sh->tmem_base, kFfnTmemCols);
        tc_fence_before();
        asm volatile("bar.arrive 1, %0;" ::"n"(kEpilogueThreads + 32) : "memory");
        __syncwarp();
        tc_fence_after();
        if (elect_one()) {
            mma_thread = true;
            const uint32_t idesc1 = idesc_f16_f32(kBM, 128);
            const uint32_t idesc2 = idesc_f16_f32(kBM, static_cast<uint32_t>(p.BN));
            const uint32_t x_addr = smem_u32(x_smem), w_addr = smem_u32(w_smem), h_addr = smem_u32(hid_smem);
            int ws = 0, xs = 0, a2 = 0;
            uint32_t wph = 0, xph = 0, a2ph = 0, c1 = 0, c2 = 0;
            bool ok = true;
            for (int t = first; ok && t < tiles; t += step) {
                if (!mbar_wait(&sh->x_full[xs], xph, &sh->abort_flag, kErrWaitMma))
                    break;
                tc_fence_after();
                if (issued == 0)
                    trace(p, kTrFirstA);
                const uint32_t xt = x_addr + static_cast<uint32_t>(xs) * x_tile_bytes;
                for (int j = 0; ok && j < nch + kFfnLag; ++j) {
                    if (j < nch) {  // GEMM1 chunk j -> acc1[c1 & 1]
                        const uint32_t b = c1 & 1u, ph = (c1 >> 1) & 1u;
                        if (!mbar_wait(&sh->acc1_empty[b], ph ^ 1u, &sh->abort_flag, kErrWaitMma)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t d = sh->tmem_base + b * 128u;
                        for (int kp = 0; kp < kpan; ++kp) {
                            if (!mbar_wait(&sh->w_full[ws], wph, &sh->abort_flag, kErrWaitMma)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            if (issued == 0)
                                trace(p, kTrWeightsLanded);
                            const uint32_t a_st = xt + static_cast<uint32_t>(kp) * kFfnPanelBytes;
                            const uint32_t b_st = w_addr + static_cast<uint32_t>(ws) * slot_bytes;
#pragma unroll
                            for (int ks = 0; ks < 4; ++ks) {
                                umma_f16(d, smem_desc(a_st + ks * 32, 16, 1024, 2), smem_desc(b_st + ks * 32, 16, 1024, 2),
                                         idesc1, (kp | ks) != 0);
                                ++issued;
                            }
                            umma_commit(&sh->w_empty[ws]);
                            if (++ws == p.b_stages) {
                                ws = 0;
                                wph ^= 1u;
                            }
                        }
                        if (!ok)
                            break;
                        umma_commit(&sh->acc1_full[b]);
                        if (c1 < 2)
                            trace(p, c1 == 0 ? kTrFfnG1First : kTrFfnG1Second);
                        if (j == nch - 1) {  // the tile's X is no longer read
                            umma_commit(&sh->x_empty[xs]);
                            if (++xs == p.a_stages) {
                                xs = 0;
                                xph ^= 1u;
                            }
                        }
                        ++c1;
                    }
                    if (j >= kFfnLag) {  // GEMM2 chunk j - kFfnLag: acc2 += hidden . W2[:, chunk]^T
                        const uint32_t hb = c2 & 1u, hph = (c2 >> 1) & 1u;
                        if (j == kFfnLag) {
                            if (!mbar_wait(&sh->acc2_empty[a2], a2ph ^ 1u, &sh->abort_flag, kErrWaitMma)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                        }
                        if (!mbar_wait(&sh->hid_full[hb], hph, &sh->abort_flag, kErrWaitMma) ||
                            !mbar_wait(&sh->w_full[ws], wph, &sh->abort_flag, kErrWaitMma)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        if (c2 == 0)
                            trace(p, kTrFfnG2First);
                        const uint32_t d2 = sh->tmem_base + 256u + static_cast<uint32_t>(a2 * p.BN);
                        const uint32_t a_st = h_addr + hb * kFfnPanelBytes;
                        const uint32_t b_st = w_addr + static_cast<uint32_t>(ws) * slot_bytes;
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks) {
                            umma_f16(d2, smem_desc(a_st + ks * 32, 16, 1024, 2), smem_desc(b_st + ks * 32, 16, 1024, 2),
                                     idesc2, (j > kFfnLag || ks > 0) ? 1u : 0u);
                            ++issued;
                        }
                        umma_commit(&sh->w_empty[ws]);
                        umma_commit(&sh->hid_empty[hb]);
                        if (++ws == p.b_stages) {
                            ws = 0;
                            wph ^= 1u;
                        }
                        ++c2;
                        if (j == nch + kFfnLag - 1) {
                            umma_commit(&sh->acc2_full[a2]);
                            if (++a2 == acc2_bufs) {
                                a2 = 0;
                                a2ph ^= 1u;
                            }
                        }
                    }
                }
            }
            trace(p, kTrLastCommit);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue warps
        const int quadrant = warp & 3;
        const int group = (warp - 2) / 4;
        const int et_id = (warp - 2) * 32 + lane;
        const int row = quadrant * 32 + lane;  // TMEM lane = pixel row of the tile
        const bool leader = et_id == 0;
        for (int i = et_id; i < 2 * fp.hidden; i += kEpilogueThreads)
            sh->bias1[i] = fp.bias1 ? __half2float(fp.bias1[i]) : 0.0f;
        for (int i = et_id; i < p.BN; i += kEpilogueThreads)
            sh->bias2[i] = (p.bias && i < p.N) ? __half2float(p.bias[i]) : 0.0f;
        asm volatile("bar.sync 1, %0;" ::"n"(kEpilogueThreads + 32) : "memory");  // biases + TMEM address
        tc_fence_after();
        pdl_wait();  // output writes follow the previous kernel
        const uint32_t lane_base = sh->tmem_base + (static_cast<uint32_t>(quadrant * 32) << 16);
        const __half2 lo2 = __float2half2_rn(p.clip_lo), hi2 = __float2half2_rn(p.clip_hi);
        const StageSync ss{&sh->stg_ready, &sh->stg_full};
        uint32_t c1 = 0, a2ph = 0, it = 0;
        int a2 = 0, xs = 0;
        bool ok = true;
        for (int t = first; ok && t < tiles; t += step, ++it) {
            // the previous tile's output stores must have read the panels
            if (leader) {
                bulk_wait_read<0>();
                mbar_arrive(ss.ready);
            }
            if (!mbar_wait(ss.ready, it & 1u, &sh->abort_flag, kErrWaitEpilogue))
                break;
            for (int j = 0; j < nch; ++j, ++c1) {
                const uint32_t b = c1 & 1u, ph = (c1 >> 1) & 1u;
                if (!mbar_wait(&sh->acc1_full[b], ph, &sh->abort_flag, kErrWaitEpilogue) ||
                    !mbar_wait(&sh->hid_empty[b], ph ^ 1u, &sh->abort_flag, kErrWaitEpilogue)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (c1 == 0 && et_id == 0)
                    trace(p, kTrFirstAcc);
                if (c1 == 1 && et_id == 0)
                    trace(p, kTrFfnChunkWaited);
                // this thread: hidden channels [32 * group, 32 * group + 32) of the chunk;
                // all 64 accumulators (32 gate, 32 linear) in one load round trip
                uint8_t* hrow = hid_smem + b * kFfnPanelBytes + row * 128;
                const float4* bg4 = reinterpret_cast<const float4*>(&sh->bias1[j * 128 + 32 * group]);
                const float4* bl4 = bg4 + 16;  // linear bias: 64 floats further
                uint32_t gr[32], lr[32];
                const uint32_t col = b * 128u + static_cast<uint32_t>(32 * group);
                tmem_ld32_nowait(lane_base + col, gr);
                tmem_ld32_nowait(lane_base + col + 64u, lr);
                tmem_wait_ld();
                if (c1 == 1 && et_id == 0)
                    trace(p, kTrFfnChunkLoaded);
                tc_fence_before();
                mbar_arrive(&sh->acc1_empty[b]);  // accumulators are in registers: GEMM1 may reuse them
                uint32_t packed[16];
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    const float4 bg = bg4[i / 4], bl = bl4[i / 4];
                    const __half2 g0 = __floats2half2_rn(__uint_as_float(gr[i]) + bg.x, __uint_as_float(gr[i + 1]) + bg.y);
                    const __half2 g1 =
                        __floats2half2_rn(__uint_as_float(gr[i + 2]) + bg.z, __uint_as_float(gr[i + 3]) + bg.w);
                    const __half2 l0 = __floats2half2_rn(__uint_as_float(lr[i]) + bl.x, __uint_as_float(lr[i + 1]) + bl.y);
                    const __half2 l1 =
                        __floats2half2_rn(__uint_as_float(lr[i + 2]) + bl.z, __uint_as_float(lr[i + 3]) + bl.w);
                    const __half2 r0 = __hmul2(__hmin2(__hmax2(g0, lo2), hi2), l0);
                    const __half2 r1 = __hmul2(__hmin2(__hmax2(g1, lo2), hi2), l1);
                    packed[i / 2] = *reinterpret_cast<const uint32_t*>(&r0);
                    packed[i / 2 + 1] = *reinterpret_cast<const uint32_t*>(&r1);
                }
                // 128-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ (r % 8)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int c = 4 * group + q;
                    *reinterpret_cast<uint4*>(hrow + ((c ^ (row & 7)) << 4)) =
                        make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
                }
                if (c1 == 1 && et_id == 0)
                    trace(p, kTrFfnChunkStored);
                fence_proxy_async_smem();  // the tensor core reads the hidden panel through the async proxy
                mbar_arrive(&sh->hid_full[b]);
                if (c1 == 1 && et_id == 0)
                    trace(p, kTrFfnChunk1Done);
                if (et_id == 0 && t == first && (j == 0 || j == nch - 1))
                    trace(p, j == 0 ? kTrFfnHidden0 : kTrFfnHiddenLast);
            }
            if (!ok)
                break;
            TileCoord tc;
            tc.pixel0 = t * kBM;
            tc.ox0 = tc.oy = 0;
            const uint8_t* x_tile = x_smem + static_cast<size_t>(xs) * x_tile_bytes;
            if (!epilogue_tile(p, sh->bias2, sh->tmem_base + 256u + static_cast<uint32_t>(a2 * p.BN), &sh->acc2_full[a2],
                               a2ph, &sh->acc2_empty[a2], ss, it, stage_smem, x_tile, p.BN / 64, 0, tc, false, quadrant,
                               group, lane, leader, &sh->abort_flag))
                break;
            if (leader && t == first)
                trace(p, kTrFfnAcc2);
            mbar_arrive(&sh->x_empty[xs]);  // residual reads of this X tile are done
            if (++xs == p.a_stages)
                xs = 0;
            if (++a2 == acc2_bufs) {
                a2 = 0;
                a2ph ^= 1u;
            }
        }
        if (leader) {
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
        tmem_dealloc(sh->tmem_base, kFfnTmemCols);
    }
    if (threadIdx.x == 0)
        trace(p, kTrExit);
}

}  // namespace mlvc_b200
