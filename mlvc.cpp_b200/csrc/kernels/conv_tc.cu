// Tensor-core convolutions for sm_100a (tcgen05 + TMEM + TMA).
//
// Both kernels compute, on channels-last (NHWC) FP16 activations,
//     out[p, n] = epilogue( sum_k A[p, k] * B[n, k] + bias[n] )
// with FP32 accumulation in tensor memory and one FP16 rounding of the conv
// result, followed by the fused operator and its own rounding, which is the
// operator-by-operator rounding of the AOT graph (reference semantics:
// backends/cpu/src/kernels_scalar.cpp:180-192; fused patterns from
// backends/driver_cubin/src/fusion_registry.cpp:711-800 and 893-1036).
//
//  * mlvc_conv1x1_tc: 1x1 conv = GEMM M = pixels, N = out channels, K = in
//    channels.  A is streamed by TMA in 128x64 panels (128-byte swizzle), the
//    whole weight slice of the CTA's N tile stays resident in shared memory.
//  * mlvc_convkxk_tc: k x k conv (stride 1 or 2, symmetric pad) as implicit
//    GEMM.  For every 64-channel slice the CTA loads ONE halo block covering
//    all taps (kh input rows x (128 + halo) pixels, interleaved 8x16-byte core
//    matrices, zero fill outside the image from the TMA bounds check) and
//    feeds every tap to the tensor core by offsetting the matrix descriptor's
//    start address by whole pixels.  Weight panels (64 channels of one tap)
//    stream through their own ring or stay resident when they fit.
//
// Warp roles (320 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA
// issuer, warps 2..9 = epilogue: two warpgroups, each warp reading its TMEM
// lane quadrant (warp % 4) and the warpgroup's share of the column chunks.  Persistent:
// each CTA walks tiles t = blockIdx.x + i * gridDim.x, and gridDim.x is a
// multiple of n_tiles so a CTA keeps one N tile.  Accumulators are double
// buffered in TMEM so the epilogue of tile i overlaps the MMAs of tile i+1.
#include "sm100.cuh"

namespace mlvc_b200 {

constexpr int kThreads = 320;          // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kEpilogueThreads = 256;  // two warpgroups, one per half of the 32-column chunks
constexpr int kBM = 128;
constexpr int kMaxStages = 8;
constexpr unsigned int kErrWaitProducer = 0x1u;
constexpr unsigned int kErrWaitMma = 0x2u;
constexpr unsigned int kErrWaitEpilogue = 0x4u;
constexpr unsigned int kErrAlign = 0x8u;

struct TcShared {
    uint64_t a_full[kMaxStages];
    uint64_t a_empty[kMaxStages];
    uint64_t b_full[kMaxStages];
    uint64_t b_empty[kMaxStages];
    uint64_t tmem_full[2];
    uint64_t tmem_empty[2];
    uint64_t stg_ready, stg_full;  // output staging hand-over (see StageSync)
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
    alignas(16) float bias[256];  // read as float2
};
static_assert(sizeof(TcShared) <= kTcHeaderBytes, "TcShared must fit the header reserved by the host");
static_assert(offsetof(TcShared, bias) % 16 == 0, "vector bias reads");

__device__ __forceinline__ void trace(const ConvTcParams& p, int point)
{
    if (p.trace)
        p.trace[blockIdx.x * kTracePoints + point] = globaltimer_ns();
}

__device__ __forceinline__ uint32_t tmem_cols_for(int bn)
{
    uint32_t need = static_cast<uint32_t>(2 * bn);
    uint32_t c = 32;
    while (c < need)
        c <<= 1;
    return c;
}

// ----------------------------------------------------------- epilogue
// The epilogue writes the whole output tile (128 rows x the tile's output
// columns) into a shared staging buffer laid out as 64-column panels of 128
// rows x 128 bytes with the 128-byte swizzle (16-byte chunk q of row r at
// chunk q ^ (r % 8)), which is exactly the shared-memory image of a {64, 128}
// SWIZZLE_128B TMA box; one thread then stores the tile with one TMA
// instruction per panel, clipped at the tensor edges.  A residual operand is
// TMA-loaded into the same buffer beforehand (or read from an operand tile
// already in shared memory in this layout).  Few TMA instructions per tile
// matter: each one occupies the SM's copy engine for tens of nanoseconds
// whatever its size.  Each epilogue warp owns one TMEM lane quadrant (32
// rows); the two warpgroups take alternate 32-column chunks.  The 32 lanes of
// a warp are 32 consecutive rows, so the 16-byte staging accesses are free of
// bank conflicts.
__device__ __forceinline__ uint32_t stage_off(int row, int col)  // col: multiple of 8 within the tile
{
    return static_cast<uint32_t>((col >> 6) * 16384 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4));
}

// TMA coordinates of an output tile: 1x1 / FFN maps are {channels, pixels},
// k x k maps are {channels, W, H}.
struct TileCoord {
    int pixel0;   // 1x1: first pixel of the tile
    int ox0, oy;  // k x k: first output column and the output row of the tile
};

__device__ __forceinline__ void tile_copy(const CUtensorMap* map, bool load, uint8_t* stage, int panels, int col0,
                                          const TileCoord& tc, bool kxk, uint64_t* bar)
{
    for (int i = 0; i < panels; ++i) {
        uint8_t* s = stage + i * 16384;
        const int x = col0 + 64 * i;
        if (load) {
            if (kxk)
                tma_load_3d(s, map, bar, x, tc.ox0, tc.oy);
            else
                tma_load_2d(s, map, bar, x, tc.pixel0);
        } else {
            if (kxk)
                tma_store_3d(map, s, x, tc.ox0, tc.oy);
            else
                tma_store_2d(map, s, x, tc.pixel0);
        }
    }
}

// Staging hand-over between tiles (both in shared memory):
//   ready: the leader thread found the previous tile's stores done reading the
//          buffer and, for a staged residual, the residual tile has landed;
//   full:  all epilogue threads wrote their rows (count kEpilogueThreads).
struct StageSync {
    uint64_t* ready;
    uint64_t* full;
};

// One thread's row of the tile: for the 32-column chunks c0 = 32 (group +
// groups k) it reads 32 accumulators, applies bias and the fused operator with
// the graph's rounding and writes the row into the staging panels.  `res` is
// the residual tile (same layout), read before the row is overwritten.
__device__ __forceinline__ void epilogue_rows(const ConvTcParams& p, const float* bias, uint32_t lane_addr, int group,
                                              int row, uint8_t* stage, const uint8_t* res, int groups)
{
    if (p.epilogue == kEpiReglu) {
        const int half = p.BN / 2;
        const __half2 lo2 = __float2half2_rn(p.clip_lo), hi2 = __float2half2_rn(p.clip_hi);
        for (int c0 = group * 32; c0 < half; c0 += 32 * groups) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t gr[16], lr[16];
                tmem_ld16_nowait(lane_addr + c0 + 16 * h, gr);
                tmem_ld16_nowait(lane_addr + half + c0 + 16 * h, lr);
                tmem_wait_ld();
                // gate/linear: FP32 bias add, one rounding each; clip and product
                // in packed FP16 (both exact on FP16 operands: the min/max select
                // and the single rounding of an exact FP16 x FP16 product equal
                // the reference's FP32 clip / multiply followed by a rounding)
                uint32_t packed[8];
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
                    const float2 bg = *reinterpret_cast<const float2*>(&bias[c0 + 16 * h + i]);
                    const float2 bl = *reinterpret_cast<const float2*>(&bias[half + c0 + 16 * h + i]);
                    const __half2 g2 = __floats2half2_rn(__uint_as_float(gr[i]) + bg.x, __uint_as_float(gr[i + 1]) + bg.y);
                    const __half2 l2 = __floats2half2_rn(__uint_as_float(lr[i]) + bl.x, __uint_as_float(lr[i + 1]) + bl.y);
                    const __half2 r2 = __hmul2(__hmin2(__hmax2(g2, lo2), hi2), l2);
                    packed[i / 2] = *reinterpret_cast<const uint32_t*>(&r2);
                }
                *reinterpret_cast<uint4*>(stage + stage_off(row, c0 + 16 * h)) =
                    make_uint4(packed[0], packed[1], packed[2], packed[3]);
                *reinterpret_cast<uint4*>(stage + stage_off(row, c0 + 16 * h + 8)) =
                    make_uint4(packed[4], packed[5], packed[6], packed[7]);
            }
        }
        return;
    }
    for (int c0 = group * 32; c0 < p.BN; c0 += 32 * groups) {
        uint32_t a[32];
        tmem_ld32_nowait(lane_addr + c0, a);
        tmem_wait_ld();
        // conv result: FP32 bias add and one rounding, packed two per register
        uint32_t h[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float2 b2 = *reinterpret_cast<const float2*>(&bias[c0 + 2 * i]);
            h[i] = pack_h2(__uint_as_float(a[2 * i]) + b2.x, __uint_as_float(a[2 * i + 1]) + b2.y);
        }
        if (p.epilogue == kEpiLeaky) {
            // negative halves become fp16(fp32(x) * alpha) (alpha is an FP32 constant)
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                float x0, x1;
                unpack_h2(h[i], x0, x1);
                const uint32_t m = pack_h2(x0 * p.alpha, x1 * p.alpha);
                const uint32_t neg = ((h[i] >> 15) & 0x00010001u) * 0xFFFFu;  // sign bit -> 16-bit mask
                h[i] = (m & neg) | (h[i] & ~neg);
            }
        } else if (p.epilogue == kEpiResidual) {
            // fp16 + fp16 with one rounding equals the FP32 add + rounding of the reference
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint4 rv = *reinterpret_cast<const uint4*>(res + stage_off(row, c0 + 8 * q));
                const uint32_t rr[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const __half2 s2 = __hadd2(*reinterpret_cast<const __half2*>(&h[4 * q + i]),
                                               *reinterpret_cast<const __half2*>(&rr[i]));
                    h[4 * q + i] = *reinterpret_cast<const uint32_t*>(&s2);
                }
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(stage + stage_off(row, c0 + 8 * q)) =
                make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
    }
}

// Leader thread, before a tile's rows are written: the stores that last used
// this staging buffer must have read it (with two buffers the previous tile's
// store may still be reading the other one); then the residual tile is loaded
// into it (load_residual) or the buffer is simply released.
__device__ __forceinline__ void stage_prepare(const ConvTcParams& p, uint8_t* stage, int panels, int col0,
                                              const TileCoord& tc, bool kxk, bool load_residual, uint64_t* ready)
{
    if (p.stage_bufs == 2)
        bulk_wait_read<1>();
    else
        bulk_wait_read<0>();
    if (load_residual) {
        mbar_arrive_expect_tx(ready, static_cast<uint32_t>(panels) * 16384u);
        tile_copy(&p.map_res, true, stage, panels, col0, tc, kxk, ready);
    } else {
        mbar_arrive(ready);
    }
}

// All epilogue threads, one tile: wait for the accumulator and the staging
// buffer, convert, release the accumulator, and let the leader store the tile.
// `it` counts the CTA's tiles (barrier parities); `groups` warps share each
// TMEM lane quadrant (column chunks split between them).  Returns false on abort.
// kShuffle: the 1x1 conv's variant that can store through the folded pixel
// shuffle (p.d2s_c); the other kernels instantiate the plain store only.
template <bool kShuffle = false>
__device__ __forceinline__ bool epilogue_tile(const ConvTcParams& p, const float* bias, uint32_t tmem_acc,
                                              uint64_t* acc_full, uint32_t acc_parity, uint64_t* acc_empty,
                                              const StageSync& ss, uint32_t it, uint8_t* stage, const uint8_t* res,
                                              int panels, int col0, const TileCoord& tc, bool kxk, int quadrant,
                                              int group, int lane, bool leader, volatile int* abort_flag,
                                              int groups = 2, int trace_at = -1)
{
    // trace_at >= 0: the leader stamps the phases of this tile at trace_at + 0..3
    const bool stamp = leader && trace_at >= 0;
    if (!mbar_wait(acc_full, acc_parity, abort_flag, kErrWaitEpilogue))
        return false;
    tc_fence_after();
    if (stamp)
        trace(p, trace_at);
    if (!mbar_wait(ss.ready, it & 1u, abort_flag, kErrWaitEpilogue))
        return false;
    if (stamp)
        trace(p, trace_at + 1);
    epilogue_rows(p, bias, tmem_acc + (static_cast<uint32_t>(quadrant * 32) << 16), group, quadrant * 32 + lane, stage,
                  res ? res : stage, groups);
    tc_fence_before();
    mbar_arrive(acc_empty);
    fence_proxy_async_smem();  // staging rows become visible to the TMA store (async proxy)
    mbar_arrive(ss.full);
    if (stamp)
        trace(p, trace_at + 2);
    if (leader) {
        if (!mbar_wait(ss.full, it & 1u, abort_flag, kErrWaitEpilogue))
            return false;
        if (stamp)
            trace(p, trace_at + 3);
        if (kShuffle && p.d2s_c) {
            // pixel shuffle folded into the store: output column n = sub * C + c
            // (sub = dy * 2 + dx) of input pixel (x, y) goes to output pixel
            // (2 x + dx, 2 y + dy), channel c; a 64-column panel never spans two
            // sub-pixels (C is a multiple of 64)
            for (int i = 0; i < panels; ++i) {
                const int n = col0 + 64 * i, sub = n / p.d2s_c;
                tma_store_5d(&p.map_out, stage + i * 16384, n - sub * p.d2s_c, sub & 1, tc.ox0, sub >> 1, tc.oy);
            }
        } else {
            tile_copy(&p.map_out, false, stage, panels, col0, tc, kxk, nullptr);
        }
        bulk_commit();
    }
    return true;
}

// kShuffle: the 1x1 conv's instantiation with the folded pixel shuffle
// (row-aligned tiles, p.row_tiles, and the 5-D store of p.d2s_c).
template <bool kShuffle = false>
__device__ __forceinline__ void epilogue_role(const ConvTcParams& p, TcShared& sh, uint8_t* stage, int warp, int lane,
                                              int n_tile, int first_tile, int tile_step, int total_tiles, bool kxk)
{
    const int quadrant = warp & 3;
    const int group = (warp - 2) / 4;          // column-chunk warpgroup
    const int et_id = (warp - 2) * 32 + lane;  // 0..255
    const bool leader = et_id == 0;
    for (int i = et_id; i < p.BN; i += kEpilogueThreads) {
        const int col = n_tile * p.BN + i;
        sh.bias[i] = (p.bias && col < p.N) ? __half2float(p.bias[col]) : 0.0f;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kEpilogueThreads + 32) : "memory");  // bias loaded + TMEM allocated
    tc_fence_after();
    pdl_wait();  // residual reads and output writes follow the previous kernel
    const int out_cols = p.epilogue == kEpiReglu ? p.BN / 2 : p.BN;
    const int panels = out_cols / 64;
    const StageSync ss{&sh.stg_ready, &sh.stg_full};
    // row-aligned tiles: k x k convs, and 1x1 convs with a folded pixel shuffle
    const int tiles_per_row = kxk ? (p.out_w + kBM - 1) / kBM : (kShuffle ? p.row_tiles : 1);
    uint32_t acc = 0, acc_phase = 0, it = 0;
    bool aborted = false;
    for (int t = first_tile; t < total_tiles; t += tile_step, ++it) {
        const int m_tile = t / p.n_tiles;
        TileCoord tc;
        tc.oy = m_tile / tiles_per_row;
        tc.ox0 = (m_tile % tiles_per_row) * kBM;
        tc.pixel0 = kShuffle ? tc.oy * p.in_w + tc.ox0 : m_tile * kBM;
        // staging buffer of this tile (two alternate when the host gave two)
        uint8_t* st = stage + (p.stage_bufs == 2 ? static_cast<size_t>(it & 1u) * panels * kTcStagePanelBytes : 0);
        if (leader)
            stage_prepare(p, st, panels, n_tile * out_cols, tc, kxk, p.epilogue == kEpiResidual, ss.ready);
        const int trace_at = it < 4 ? kTrConvEpi + 4 * static_cast<int>(it) : -1;
        const bool tile_ok =
            epilogue_tile<kShuffle>(p, sh.bias, sh.tmem_base + acc * p.BN, &sh.tmem_full[acc], acc_phase,
                                    &sh.tmem_empty[acc], ss, it, st, nullptr, panels, n_tile * out_cols, tc, kxk,
                                    quadrant, group, lane, leader, &sh.abort_flag, 2, trace_at);
        if (!tile_ok) {
            aborted = true;
            break;
        }
        if (leader && it < 4)
            trace(p, kTrConvTile + 4 * static_cast<int>(it) + 2);
        if (t == first_tile && leader)
            trace(p, kTrFirstAcc);
        acc ^= 1u;
        acc_phase ^= (acc == 0) ? 1u : 0u;
    }
    if (leader) {
        // On abort, a residual tile this leader loaded for tile `it` may still
        // be in flight: wait (bounded) for its barrier phase before the CTA's
        // shared memory retires.  When the phase already completed, the wait
        // returns at once.
        if (aborted && p.epilogue == kEpiResidual) {
            volatile int never = 0;
            mbar_wait(ss.ready, it & 1u, &never, kErrWaitEpilogue);
        }
        bulk_wait_all();  // stores complete before the CTA (and its shared memory) retires
        trace(p, kTrEpilogueDone);
    }
}

// --------------------------------------------------------------- setup
__device__ __forceinline__ TcShared* setup_shared(uint8_t* smem_raw, const ConvTcParams& p, int warp)
{
    TcShared* sh = reinterpret_cast<TcShared*>(smem_raw);
    if (threadIdx.x == 0)
        trace(p, kTrEntry);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kMaxStages; ++s) {
            mbar_init(&sh->a_full[s], 1);
            mbar_init(&sh->a_empty[s], 1);
            mbar_init(&sh->b_full[s], 1);
            mbar_init(&sh->b_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&sh->tmem_full[s], 1);
            mbar_init(&sh->tmem_empty[s], kEpilogueThreads);
        }
        mbar_init(&sh->stg_ready, 1);
        mbar_init(&sh->stg_full, kEpilogueThreads);
        mbar_init(&sh->drain, 1);
        sh->abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && elect_one()) {
        tma_prefetch_desc(&p.map_a0);
        if (p.a_split)
            tma_prefetch_desc(&p.map_a1);
        tma_prefetch_desc(&p.map_b);
        tma_prefetch_desc(&p.map_out);
        if (p.epilogue == kEpiResidual)
            tma_prefetch_desc(&p.map_res);
    }
    // Only the barriers must be visible before the producer starts; TMEM is
    // allocated by warp 1 afterwards and handed to the epilogue warps through
    // named barrier 1 (see alloc_tmem_and_publish / epilogue_role).
    __syncthreads();
    if (threadIdx.x == 0)
        trace(p, kTrSetup);
    pdl_launch_dependents();
    return sh;
}

// Warp 1: allocate the accumulators and publish their address to the
// epilogue warpgroups (named barrier 1: 256 epilogue threads + this warp).
__device__ __forceinline__ void alloc_tmem_and_publish(TcShared* sh, const ConvTcParams& p)
{
    tmem_alloc(&sh->tmem_base, tmem_cols_for(p.BN));
    tc_fence_before();
    asm volatile("bar.arrive 1, %0;" ::"n"(kEpilogueThreads + 32) : "memory");
    __syncwarp();
    tc_fence_after();
}

__device__ __forceinline__ void teardown(const ConvTcParams& p, TcShared* sh, int warp, bool mma_thread,
                                         uint32_t issued_mma)
{
    // An aborted MMA issuer drains its outstanding tcgen05.mma before TMEM is freed.
    if (mma_thread && sh->abort_flag && issued_mma) {
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

// Register-resident record of the TMA loads a producer armed: bit s of
// `armed` = slot s was armed, bit s of `parity` = the phase it was armed for
// (bit masks rather than arrays, so nothing of it lives in local memory).
struct ArmedSlots {
    uint32_t armed = 0, parity = 0;
    __device__ __forceinline__ void arm(int s, uint32_t phase)
    {
        armed |= 1u << s;
        parity = (parity & ~(1u << s)) | (phase << s);
    }
};

// Producer-side drain: wait (bounded) for every TMA this thread armed, so no
// bulk copy is still writing shared memory when an aborted CTA exits.
__device__ __forceinline__ void drain_armed(uint64_t* bars, const ArmedSlots& a, int n)
{
    volatile int never = 0;
    for (int s = 0; s < n; ++s)
        if ((a.armed >> s) & 1u)
            mbar_wait(&bars[s], (a.parity >> s) & 1u, &never, kErrWaitProducer);
}

// ===================================================== 1x1 conv (GEMM)
template <bool kShuffle>
__device__ __forceinline__ void conv1x1_tc(const ConvTcParams& p)
{
    extern __shared__ __align__(1024) uint8_t smem_dyn[];
    // 1024-byte alignment for the swizzled operand tiles.
    uint8_t* base = align_smem_1024(smem_dyn);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    TcShared* sh = setup_shared(base, p, warp);
    uint8_t* b_smem = base + ((sizeof(TcShared) + 1023) & ~size_t(1023));
    const int k_panels = (p.K + 63) / 64;  // channels past K read as TMA zero fill
    const size_t b_panel_bytes = static_cast<size_t>(p.BN) * 128;
    uint8_t* a_smem = b_smem + b_panel_bytes * k_panels;
    constexpr uint32_t kAPanelBytes = kBM * 128;
    uint8_t* stage_smem = a_smem + static_cast<size_t>(p.a_stages) * kAPanelBytes;  // 1024-aligned

    const int total_tiles = p.m_tiles * p.n_tiles;
    const int n_tile = blockIdx.x % p.n_tiles;
    const int first = blockIdx.x, step = gridDim.x;
    bool mma_thread = false;
    uint32_t issued = 0;

    if (warp == 0) {
        if (elect_one()) {
            ArmedSlots a_armed, b_armed;
            b_armed.arm(0, 0);
            mbar_arrive_expect_tx(&sh->b_full[0], static_cast<uint32_t>(b_panel_bytes * k_panels));
            for (int kp = 0; kp < k_panels; ++kp)
                tma_load_2d(b_smem + kp * b_panel_bytes, &p.map_b, &sh->b_full[0], kp * 64, n_tile * p.BN);
            trace(p, kTrWeightsIssued);
            pdl_wait();  // activations are written by the previous kernel
            trace(p, kTrDepReady);
            int stage = 0;
            uint32_t phase = 0;
            int panel = 0;  // A panels this CTA has handled (wait-expiry test)
            const int withhold = blockIdx.x == 0 ? p.withhold_a : 0;
            for (int t = first; t < total_tiles && !sh->abort_flag; t += step) {
                const int m_tile = t / p.n_tiles;
                // first pixel of the tile (row-aligned tiles: row m_tile / row_tiles)
                const int pixel0 = kShuffle ? (m_tile / p.row_tiles) * p.in_w + (m_tile % p.row_tiles) * kBM
                                               : m_tile * kBM;
                for (int kp = 0; kp < k_panels; ++kp) {
                    if (!mbar_wait(&sh->a_empty[stage], phase ^ 1u, &sh->abort_flag, kErrWaitProducer))
                        break;
                    if (++panel != withhold) {
                        mbar_arrive_expect_tx(&sh->a_full[stage], kAPanelBytes);
                        // K panels past a_split come from the second tensor of a concat
                        const bool second = p.a_split > 0 && kp >= p.a_split;
                        tma_load_2d(a_smem + stage * kAPanelBytes, second ? &p.map_a1 : &p.map_a0,
                                    &sh->a_full[stage], (second ? kp - p.a_split : kp) * 64, pixel0);
                        a_armed.arm(stage, phase);
                    }
                    if (++stage == p.a_stages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (sh->abort_flag) {
                drain_armed(sh->a_full, a_armed, p.a_stages);
                drain_armed(sh->b_full, b_armed, 1);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        alloc_tmem_and_publish(sh, p);
        if (elect_one()) {
            mma_thread = true;
            const uint32_t idesc = idesc_f16_f32(kBM, static_cast<uint32_t>(p.BN));
            if (mbar_wait(&sh->b_full[0], 0, &sh->abort_flag, kErrWaitMma)) {
                tc_fence_after();
                trace(p, kTrWeightsLanded);
                int stage = 0;
                uint32_t phase = 0, acc = 0, acc_phase = 0;
                const uint32_t b_addr = smem_u32(b_smem), a_addr = smem_u32(a_smem);
                int tile_no = 0;
                for (int t = first; t < total_tiles; t += step, ++tile_no) {
                    if (!mbar_wait(&sh->tmem_empty[acc], acc_phase ^ 1u, &sh->abort_flag, kErrWaitMma))
                        break;
                    tc_fence_after();
                    if (tile_no < 4)
                        trace(p, kTrConvTile + 4 * tile_no);
                    const uint32_t d = sh->tmem_base + acc * static_cast<uint32_t>(p.BN);
                    bool ok = true;
                    for (int kp = 0; kp < k_panels; ++kp) {
                        if (!mbar_wait(&sh->a_full[stage], phase, &sh->abort_flag, kErrWaitMma)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        if (issued == 0)
                            trace(p, kTrFirstA);
                        const uint32_t a_st = a_addr + stage * kAPanelBytes;
                        const uint32_t b_st = b_addr + static_cast<uint32_t>(kp * b_panel_bytes);
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks) {
                            const uint64_t ad = smem_desc(a_st + ks * 32, 16, 1024, 2);
                            const uint64_t bd = smem_desc(b_st + ks * 32, 16, 1024, 2);
                            umma_f16(d, ad, bd, idesc, (kp | ks) != 0);
                            ++issued;
                        }
                        umma_commit(&sh->a_empty[stage]);
                        if (++stage == p.a_stages) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (!ok)
                        break;
                    umma_commit(&sh->tmem_full[acc]);
                    if (tile_no < 4)
                        trace(p, kTrConvTile + 4 * tile_no + 1);
                    acc ^= 1u;
                    acc_phase ^= (acc == 0) ? 1u : 0u;
                }
                trace(p, kTrLastCommit);
            }
        }
        __syncwarp();
    } else {
        epilogue_role<kShuffle>(p, *sh, stage_smem, warp, lane, n_tile, first, step, total_tiles, false);
    }
    teardown(p, sh, warp, mma_thread, issued);
}

extern "C" __global__ void __launch_bounds__(kThreads, 2) mlvc_conv1x1_tc(const __grid_constant__ ConvTcParams p)
{
    conv1x1_tc<false>(p);
}

// the same GEMM with a 2x pixel shuffle folded into its store (see ConvTcParams::d2s_c)
extern "C" __global__ void __launch_bounds__(kThreads, 2) mlvc_conv1x1_d2s_tc(const __grid_constant__ ConvTcParams p)
{
    conv1x1_tc<true>(p);
}

// ===================================================== k x k conv
// Halo layout in shared memory for one 64-channel slice:
//   [parity q][chunk j (8 channels)][row r][pixel x] x 16 bytes
// so that for a fixed (q, row) the pixels of one chunk sit at a 16-byte
// stride (the rows of an interleaved core matrix) and consecutive chunks are
// LBO = kh * halo_px * 16 bytes apart.
extern "C" __global__ void __launch_bounds__(kThreads, 1) mlvc_convkxk_tc(const __grid_constant__ ConvTcParams p)
{
    extern __shared__ __align__(1024) uint8_t smem_dyn[];
    uint8_t* base = align_smem_1024(smem_dyn);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    TcShared* sh = setup_shared(base, p, warp);
    if (warp == 0 && elect_one() && p.stride == 2)
        tma_prefetch_desc(&p.map_a1);

    const int parities = p.stride;  // 1 or 2 halo views
    const int k_panels = p.in_c / 64;
    const int taps = p.kh * p.kw;
    // One chunk = kh rows x halo_px pixels x 16 bytes written by one TMA copy;
    // chunk starts are padded to 128 bytes (the TMA destination alignment) and
    // that padded stride is the descriptor's leading byte offset.
    const uint32_t chunk_payload = static_cast<uint32_t>(p.kh * p.halo_px * 16);
    const uint32_t chunk_bytes = (chunk_payload + 127u) & ~127u;  // LBO
    const uint32_t halo_tx = static_cast<uint32_t>(parities * 8) * chunk_payload;
    const uint32_t halo_bytes = static_cast<uint32_t>(parities * 8) * chunk_bytes;
    const uint32_t halo_stride = (halo_bytes + 1023u) & ~1023u;
    const uint32_t b_panel_bytes = static_cast<uint32_t>(p.BN) * 128u;
    uint8_t* b_smem = base + ((sizeof(TcShared) + 1023) & ~size_t(1023));
    const int b_slots = p.b_resident ? taps * k_panels : p.b_stages;
    uint8_t* a_smem = b_smem + static_cast<size_t>(b_slots) * b_panel_bytes;
    uint8_t* stage_smem = a_smem + static_cast<size_t>(p.a_stages) * halo_stride;  // 1024-aligned

    const int tiles_per_row = (p.out_w + kBM - 1) / kBM;
    const int total_tiles = p.m_tiles * p.n_tiles;
    const int n_tile = blockIdx.x % p.n_tiles;
    const int first = blockIdx.x, step = gridDim.x;
    bool mma_thread = false;
    uint32_t issued = 0;

    if (warp == 0) {
        if (elect_one()) {
            ArmedSlots a_armed, b_armed;
            if (p.b_resident) {
                mbar_arrive_expect_tx(&sh->b_full[0], b_panel_bytes * taps * k_panels);
                for (int kp = 0; kp < k_panels; ++kp)
                    for (int tap = 0; tap < taps; ++tap)
                        tma_load_2d(b_smem + static_cast<size_t>(kp * taps + tap) * b_panel_bytes, &p.map_b,
                                    &sh->b_full[0], tap * p.in_c + kp * 64, n_tile * p.BN);
                b_armed.arm(0, 0);
            }
            pdl_wait();  // activations are written by the previous kernel
            trace(p, kTrDepReady);
            int as = 0, bs = 0;
            uint32_t aph = 0, bph = 0;
            for (int t = first; t < total_tiles && !sh->abort_flag; t += step) {
                const int m_tile = t / p.n_tiles;
                const int oy = m_tile / tiles_per_row;
                const int ox0 = (m_tile % tiles_per_row) * kBM;
                const int iy0 = oy * p.stride - p.pad;
                // first halo pixel (stride 1) or pixel pair (stride 2)
                const int x0 = (p.stride == 1) ? ox0 - p.pad : ox0 + p.px_min;
                for (int kp = 0; kp < k_panels; ++kp) {
                    if (!mbar_wait(&sh->a_empty[as], aph ^ 1u, &sh->abort_flag, kErrWaitProducer))
                        break;
                    uint8_t* dst = a_smem + static_cast<size_t>(as) * halo_stride;
                    if (smem_u32(dst) & 127u) {  // never expected: refuse rather than fault
                        atomicOr(&mlvc_b200_status, kErrAlign);
                        sh->abort_flag = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&sh->a_full[as], halo_tx);
                    for (int q = 0; q < parities; ++q)
                        for (int j = 0; j < 8; ++j)
                            tma_load_3d(dst + (q * 8 + j) * chunk_bytes, q ? &p.map_a1 : &p.map_a0, &sh->a_full[as],
                                        kp * 64 + j * 8, x0, iy0);
                    a_armed.arm(as, aph);
                    if (++as == p.a_stages) {
                        as = 0;
                        aph ^= 1u;
                    }
                    if (!p.b_resident) {
                        for (int tap = 0; tap < taps; ++tap) {
                            if (!mbar_wait(&sh->b_empty[bs], bph ^ 1u, &sh->abort_flag, kErrWaitProducer))
                                break;
                            mbar_arrive_expect_tx(&sh->b_full[bs], b_panel_bytes);
                            tma_load_2d(b_smem + static_cast<size_t>(bs) * b_panel_bytes, &p.map_b, &sh->b_full[bs],
                                        tap * p.in_c + kp * 64, n_tile * p.BN);
                            b_armed.arm(bs, bph);
                            if (++bs == p.b_stages) {
                                bs = 0;
                                bph ^= 1u;
                            }
                        }
                    }
                }
            }
            if (sh->abort_flag) {
                drain_armed(sh->a_full, a_armed, p.a_stages);
                drain_armed(sh->b_full, b_armed, p.b_resident ? 1 : p.b_stages);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        alloc_tmem_and_publish(sh, p);
        if (elect_one()) {
            mma_thread = true;
            const uint32_t idesc = idesc_f16_f32(kBM, static_cast<uint32_t>(p.BN));
            bool ok = true;
            if (p.b_resident)
                ok = mbar_wait(&sh->b_full[0], 0, &sh->abort_flag, kErrWaitMma);
            int as = 0, bs = 0;
            uint32_t aph = 0, bph = 0, acc = 0, acc_phase = 0;
            const uint32_t a_addr = smem_u32(a_smem), b_addr = smem_u32(b_smem);
            for (int t = first; ok && t < total_tiles; t += step) {
                if (!mbar_wait(&sh->tmem_empty[acc], acc_phase ^ 1u, &sh->abort_flag, kErrWaitMma))
                    break;
                tc_fence_after();
                const uint32_t d = sh->tmem_base + acc * static_cast<uint32_t>(p.BN);
                bool first_mma = true;
                for (int kp = 0; ok && kp < k_panels; ++kp) {
                    if (!mbar_wait(&sh->a_full[as], aph, &sh->abort_flag, kErrWaitMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t halo = a_addr + as * halo_stride;
                    for (int ky = 0; ok && ky < p.kh; ++ky) {
                        for (int kx = 0; kx < p.kw; ++kx) {
                            const int tap = ky * p.kw + kx;
                            uint32_t b_panel;
                            if (p.b_resident) {
                                b_panel = b_addr + static_cast<uint32_t>(kp * taps + tap) * b_panel_bytes;
                            } else {
                                if (!mbar_wait(&sh->b_full[bs], bph, &sh->abort_flag, kErrWaitMma)) {
                                    ok = false;
                                    break;
                                }
                                tc_fence_after();
                                b_panel = b_addr + bs * b_panel_bytes;
                            }
                            int q, xoff;
                            if (p.stride == 1) {
                                q = 0;
                                xoff = kx;
                            } else {
                                const int dlt = kx - p.pad;                 // input offset of this tap
                                q = dlt & 1;                                 // parity (two's complement)
                                xoff = ((dlt - q) >> 1) - p.px_min;          // pair offset inside the halo
                            }
                            const uint32_t a_tap = halo + static_cast<uint32_t>(q * 8) * chunk_bytes +
                                                   static_cast<uint32_t>(ky * p.halo_px + xoff) * 16u;
#pragma unroll
                            for (int ks = 0; ks < 4; ++ks) {
                                const uint64_t ad = smem_desc(a_tap + ks * 2 * chunk_bytes, chunk_bytes, 128, 0);
                                const uint64_t bd = smem_desc(b_panel + ks * 32, 16, 1024, 2);
                                umma_f16(d, ad, bd, idesc, first_mma ? 0u : 1u);
                                first_mma = false;
                                ++issued;
                            }
                            if (!p.b_resident) {
                                umma_commit(&sh->b_empty[bs]);
                                if (++bs == p.b_stages) {
                                    bs = 0;
                                    bph ^= 1u;
                                }
                            }
                        }
                    }
                    umma_commit(&sh->a_empty[as]);
                    if (++as == p.a_stages) {
                        as = 0;
                        aph ^= 1u;
                    }
                }
                if (!ok)
                    break;
                umma_commit(&sh->tmem_full[acc]);
                acc ^= 1u;
                acc_phase ^= (acc == 0) ? 1u : 0u;
            }
        }
        __syncwarp();
    } else {
        epilogue_role(p, *sh, stage_smem, warp, lane, n_tile, first, step, total_tiles, true);
    }
    teardown(p, sh, warp, mma_thread, issued);
}

}  // namespace mlvc_b200
