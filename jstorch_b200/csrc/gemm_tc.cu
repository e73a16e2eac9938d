// gemm_tc.cu -- split-precision (3 x TF32) fp32 GEMM on the sm_100a tensor
// cores (tcgen05.mma kind::tf32, accumulator in TMEM, operands staged by TMA).
//
// Replaces the cuBLAS sgemm of native/ops/matmul.cu:35-36 / :48-49 / :61-62,
// which runs single-pass TF32 (matmul.cu:12).  Here each fp32 operand x is
// split into hi = rn_tf32(x) and lo = rn_tf32(x - hi), and
//     A*B ~= A_lo*B_hi + A_hi*B_lo + A_hi*B_hi
// is accumulated in fp32 in TMEM (the dropped A_lo*B_lo term is below 2^-22
// relative per product), which keeps the result within the fp32 interface's
// tolerance while running on the tensor pipe.
//
// Two kernels:
//   split_*      one HBM pass over each operand: writes hi and lo planes in a
//                K-major layout [batch][rows][Kp] (Kp = K rounded up to 4, so
//                rows are 16-byte aligned for TMA).  This pass also absorbs
//                the NN / NT / TN layouts: an MN-major operand is transposed
//                through shared memory on the way.
//   tc_gemm      warp-specialised pipeline per 128 x 256 output tile:
//                  warp 0      TMA producer: 4 tiles (A_hi, A_lo, B_hi, B_lo)
//                              per 16-wide k-slab, swizzle-64B, into a
//                              4-stage shared-memory ring
//                  warp 1      allocates 512 TMEM columns (two accumulators);
//                              one thread issues 6 tcgen05.mma (2 k-steps x 3
//                              products) per slab and commits each slab back to
//                              the producer
//                  warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns,
//                              fused bias / ReLU, a shared-memory transpose,
//                              then row-contiguous 128-byte stores to C
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "gemm_internal.h"
#include "ptx.cuh"

namespace jst {

namespace tc {

constexpr int BM = 128;
constexpr int BK = 16;  // fp32 elements per k-slab: 64-byte rows, swizzle-64B
constexpr int THREADS = 192;
// Epilogue staging: each of the 4 epilogue warps transposes its 32 x 32 fp32
// block through shared memory (rows 36 floats apart: 16-byte aligned and
// bank-conflict free for the float4 accesses) so that every store instruction
// writes four full 128-byte row segments of C.
constexpr int STG_LD = 36;
constexpr uint32_t STG_BYTES = 4 * 32 * STG_LD * 4;  // 18 KiB

// Tile configurations: BN columns of C per CTA, STAGES-deep TMA ring.
// Two fp32 accumulators of 128 lanes x BN columns: D_hi receives only the
// A_hi*B_hi products, D_lo the two small cross products.  The tensor core's
// fp32 accumulation truncates each add relative to the accumulator's own
// magnitude, so keeping the ~2^-11 smaller cross terms out of D_hi cuts the
// number of truncating adds into the large accumulator by three.
//   BN = 256, 4 stages: 512 TMEM columns, 193 KiB of shared memory, one CTA
//     per SM -- the large-GEMM configuration;
//   BN = 128, 3 stages and BN = 64, 4 stages: 256 / 128 TMEM columns and
//     97 KiB, so two CTAs share an SM and one's epilogue overlaps the other's
//     main loop -- for narrow outputs (N <= 128) and short K, where a lone CTA
//     spends most of its time outside the MMA loop or waiting on memory.
template <int BN_, int STAGES_>
struct Cfg {
    static constexpr int BN = BN_;
    static constexpr int STAGES = STAGES_;
    static constexpr uint32_t TMEM_COLS = BN_ == 256 ? 512 : (BN_ == 128 ? 256 : 128);
    static constexpr uint32_t D_HI_COL = 0;
    static constexpr uint32_t D_LO_COL = BN_;
    static constexpr uint32_t A_TILE_BYTES = BM * BK * 4;
    static constexpr uint32_t B_TILE_BYTES = BN_ * BK * 4;
    static constexpr uint32_t STAGE_BYTES = 2 * A_TILE_BYTES + 2 * B_TILE_BYTES;
    static constexpr uint32_t RING_BYTES = STAGES_ * STAGE_BYTES;
    // The epilogue's staging tiles reuse the start of the ring: by the time the
    // accumulator is complete every TMA write and tensor-core read of the ring
    // has finished.
    static_assert(RING_BYTES >= STG_BYTES, "staging aliases the ring");
    static constexpr uint32_t SMEM_BYTES = RING_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;
    static constexpr int MIN_BLOCKS = SMEM_BYTES <= 113 * 1024 ? 2 : 1;
    static_assert(2 * BN_ <= (int)TMEM_COLS, "accumulators must fit the TMEM allocation");
    static_assert(STAGES_ * 3 + 1 <= 30, "barrier area");
};
using CfgWide = Cfg<256, 4>;
using CfgMid = Cfg<128, 3>;
using CfgNarrow = Cfg<64, 4>;

struct Params {
    int M, N, K, batch;
    float* C;
    int64_t ldc, strideC;
    const float* bias;
    int bias_row;  // bias[row] instead of bias[col]
    int relu;
    int tiles_m, tiles_n;
    uint32_t* err;  // device error word
    int mc_store;   // C is a multicast address: store with multimem.st (fused all-gather)
    const float* aux;  // mask epilogue: C *= (aux > 0)
    int64_t ld_aux, stride_aux;
    int a_bcast, b_bcast;  // operand planes hold one batch entry shared by every batch
    int kslices;           // > 1: split K; C receives partials [slice][batch][M][N]
    int kb_per_slice;      // BK steps per slice
    int split_a;           // tm_a_hi maps the raw fp32 A; the epilogue warps split it in shared memory
    int tma_store;         // persistent kernel: C is written by TMA stores through tm_c
};

__device__ __forceinline__ float epi(float v, const float* bias, int col, int relu) {
    if (bias) v += __ldg(bias + col);
    if (relu) v = fmaxf(v, 0.0f);
    return v;
}

template <class C>
__global__ void __launch_bounds__(THREADS, C::MIN_BLOCKS)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tm_a_hi, const __grid_constant__ CUtensorMap tm_a_lo,
                   const __grid_constant__ CUtensorMap tm_b_hi, const __grid_constant__ CUtensorMap tm_b_lo,
                   const Params p) {
    constexpr int BN = C::BN;
    constexpr int STAGES = C::STAGES;
    constexpr uint32_t TMEM_COLS = C::TMEM_COLS, D_HI_COL = C::D_HI_COL, D_LO_COL = C::D_LO_COL;
    constexpr uint32_t A_TILE_BYTES = C::A_TILE_BYTES, B_TILE_BYTES = C::B_TILE_BYTES;
    constexpr uint32_t STAGE_BYTES = C::STAGE_BYTES, RING_BYTES = C::RING_BYTES;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment keeps every tile on a swizzle-pattern boundary
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + RING_BYTES);
    uint64_t* empty_bar = full_bar + STAGES;
    uint64_t* conv_bar = empty_bar + STAGES;  // split_a: the stage's A tile has been split
    uint64_t* accum_bar = conv_bar + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_bar + 1);
    volatile uint32_t* err = tmem_slot + 1;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // grouped rasterisation: bands of 16 tile-rows, so a wave of 148 CTAs
    // covers about 16 x 9 tiles and the concurrently running CTAs share their
    // A and B k-slabs in L2 (bands of 8 read 27 % more from DRAM at 8192^3)
    // CTA index = ((bidx * kslices) + slice) * tiles + tile: the CTAs of one
    // K slice run next to each other and share its operand panels in L2
    const int tiles_per_batch = p.tiles_m * p.tiles_n;
    const int t = blockIdx.x % tiles_per_batch;
    const int zs = blockIdx.x / tiles_per_batch;
    const int slice = zs % p.kslices;
    const int bidx = zs / p.kslices;
    constexpr int GROUP = 16;
    const int group_span = GROUP * p.tiles_n;
    const int g = t / group_span;
    const int first_m = g * GROUP;
    const int gm = min(p.tiles_m - first_m, GROUP);
    const int tm = first_m + (t % group_span) % gm;
    const int tn_band = (t % group_span) / gm;
    // Wide tiles (one CTA per SM, so a wave is 148 consecutive CTAs): the
    // waves of a band share their A panels, which are larger than L2.  The
    // CTAs of odd waves walk K downwards, so a wave starts on the k-slabs the
    // previous wave read last and still finds them in L2, while the CTAs of
    // one wave keep moving through K together (sharing their k-slabs); odd
    // bands walk the tile columns backwards, so a band starts on the B panels
    // the previous band ended on.  Each output still sums its K steps in one
    // fixed order (set by its CTA index), so results repeat bit for bit.
    constexpr int WAVE = 148;
    const bool wide_order = BN == 256 && p.kslices == 1;
    const int tn = (wide_order && (g & 1)) ? p.tiles_n - 1 - tn_band : tn_band;
    const bool k_down = wide_order && ((blockIdx.x / WAVE) & 1);
    const int m0 = tm * BM;
    const int n0 = tn * BN;
    const int kb0 = slice * p.kb_per_slice;  // this CTA's K steps: [kb0, kb0 + num_kb)
    const int num_kb = min((p.K + BK - 1) / BK - kb0, p.kb_per_slice);
    const int za = p.a_bcast ? 0 : bidx, zb = p.b_bcast ? 0 : bidx;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full_bar[s], 1);
            ptx::mbar_init(&empty_bar[s], 1);
            ptx::mbar_init(&conv_bar[s], 4);  // one arrival per splitting warp
        }
        ptx::mbar_init(accum_bar, 1);
        *err = 0;
        ptx::fence_barrier_init();
        ptx::tma_prefetch_desc(&tm_a_hi);
        ptx::tma_prefetch_desc(&tm_a_lo);
        ptx::tma_prefetch_desc(&tm_b_hi);
        ptx::tma_prefetch_desc(&tm_b_lo);
    }
    if (warp == 1) ptx::tmem_alloc<TMEM_COLS>(tmem_slot);
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Launched as a programmatic dependent (pdl), the set-up above overlapped
    // the previous kernel; no global memory is touched before this wait.
    ptx::griddep_wait();
    ptx::griddep_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ TMA producer
            for (int kb = 0; kb < num_kb; ++kb) {
                const int s = kb % STAGES;
                const uint32_t phase = (kb / STAGES) & 1;
                if (!ptx::mbar_wait(&empty_bar[s], phase ^ 1, err)) break;
                uint8_t* st = smem + s * STAGE_BYTES;
                ptx::mbar_arrive_expect_tx(&full_bar[s], p.split_a ? STAGE_BYTES - A_TILE_BYTES : STAGE_BYTES);
                const int kx = (kb0 + (k_down ? num_kb - 1 - kb : kb)) * BK;
                ptx::tma_load_3d(st, &tm_a_hi, &full_bar[s], kx, m0, za);  // split_a: the raw fp32 tile
                if (!p.split_a) ptx::tma_load_3d(st + A_TILE_BYTES, &tm_a_lo, &full_bar[s], kx, m0, za);
                ptx::tma_load_3d(st + 2 * A_TILE_BYTES, &tm_b_hi, &full_bar[s], kx, n0, zb);
                ptx::tma_load_3d(st + 2 * A_TILE_BYTES + B_TILE_BYTES, &tm_b_lo, &full_bar[s], kx, n0, zb);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------ MMA issuer
            constexpr uint32_t idesc = ptx::idesc_tf32(BM, BN);
            bool ok = true;
            for (int kb = 0; kb < num_kb && ok; ++kb) {
                const int s = kb % STAGES;
                const uint32_t phase = (kb / STAGES) & 1;
                if (!ptx::mbar_wait(p.split_a ? &conv_bar[s] : &full_bar[s], phase, err)) { ok = false; break; }
                ptx::tc_fence_after();
                const uint32_t st = ptx::smem_u32(smem + s * STAGE_BYTES);
                const uint32_t a_hi = st, a_lo = st + A_TILE_BYTES;
                const uint32_t b_hi = st + 2 * A_TILE_BYTES, b_lo = b_hi + B_TILE_BYTES;
#pragma unroll
                for (int kk = 0; kk < BK / 8; ++kk) {  // 8 tf32 = 32 bytes per MMA
                    const uint32_t off = kk * 32;
                    const uint32_t acc0 = (kb | kk) != 0;
                    const uint64_t dah = ptx::smem_desc_kmajor(a_hi + off, 64);
                    const uint64_t dbh = ptx::smem_desc_kmajor(b_hi + off, 64);
                    ptx::mma_tf32(tmem_base + D_LO_COL, ptx::smem_desc_kmajor(a_lo + off, 64), dbh, idesc, acc0);
                    ptx::mma_tf32(tmem_base + D_LO_COL, dah, ptx::smem_desc_kmajor(b_lo + off, 64), idesc, 1);
                    ptx::mma_tf32(tmem_base + D_HI_COL, dah, dbh, idesc, acc0);
                }
                ptx::mma_commit(&empty_bar[s]);  // slot s is free once these MMAs finish
            }
            ptx::mma_commit(accum_bar);  // always signalled, also on the error path
        }
    } else {
        // ---------------------------------------------------- A split (split_a)
        // The TMA wrote the raw fp32 A tile into the A_hi slot with the same
        // swizzled placement the hi / lo planes would have, so the split is
        // elementwise at unchanged offsets: hi in place, lo into the A_lo
        // slot.  fence.proxy.async makes these generic stores visible to the
        // tensor core before the warp's arrival releases the MMA issuer.
        if (p.split_a) {
            const int ct = threadIdx.x - 64;  // 0..127
            for (int kb = 0; kb < num_kb; ++kb) {
                const int s = kb % STAGES;
                const uint32_t phase = (kb / STAGES) & 1;
                int okw = 0;
                if (lane == 0) okw = ptx::mbar_wait(&full_bar[s], phase, err);
                if (!__shfl_sync(0xffffffffu, okw, 0)) break;
                float4* hi = reinterpret_cast<float4*>(smem + s * STAGE_BYTES);
                float4* lo = reinterpret_cast<float4*>(smem + s * STAGE_BYTES + A_TILE_BYTES);
#pragma unroll
                for (int i = 0; i < (int)(A_TILE_BYTES / 16) / 128; ++i) {
                    const int idx = ct + i * 128;
                    const float4 v = hi[idx];
                    float4 h, l;
                    h.x = ptx::to_tf32(v.x); l.x = ptx::to_tf32(v.x - h.x);
                    h.y = ptx::to_tf32(v.y); l.y = ptx::to_tf32(v.y - h.y);
                    h.z = ptx::to_tf32(v.z); l.z = ptx::to_tf32(v.z - h.z);
                    h.w = ptx::to_tf32(v.w); l.w = ptx::to_tf32(v.w - h.w);
                    hi[idx] = h;
                    lo[idx] = l;
                }
                ptx::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(&conv_bar[s]);
            }
        }
        // ---------------------------------------------------- epilogue
        // one lane waits and broadcasts, so the warp stays converged for the
        // .sync.aligned TMEM loads below
        int okw = 0;
        if (lane == 0) okw = ptx::mbar_wait(accum_bar, 0, err) && *err == 0;
        const bool ok = __shfl_sync(0xffffffffu, okw, 0) != 0;
        ptx::tc_fence_after();
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const int row = m0 + q * 32 + lane;
        const bool row_ok = ok && row < p.M;
        float* cbase = p.C + (int64_t)(p.kslices > 1 ? slice * p.batch + bidx : bidx) * p.strideC;
        float* crow = cbase + (int64_t)row * p.ldc;
        const bool vec = ((p.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
                         ((p.strideC & 3) == 0);
        float* stg = reinterpret_cast<float*>(smem) + (warp - 2) * (32 * STG_LD);  // aliases ring stage 0
        // a row bias is added in registers before epi(); epi() then sees no column bias
        const bool row_bias = p.bias_row && p.bias;
        const float* cbias = p.bias_row ? nullptr : p.bias;
        const float rbias = (row_bias && row < p.M) ? __ldg(p.bias + row) : 0.0f;
        if (ok) {
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                const int col0 = n0 + c * 32;
                if (col0 >= p.N) break;  // warp-uniform
                uint32_t r[32], rl[32];
                const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32);
                ptx::tmem_ld_32x32b_x32(taddr + D_HI_COL, r);
                ptx::tmem_ld_32x32b_x32(taddr + D_LO_COL, rl);
                ptx::tmem_ld_wait();
                // A non-finite D_hi (an Inf or NaN operand, or overflow) is the
                // result: D_lo then holds Inf * 0 = NaN from the cross terms of
                // an infinite operand (its lo part is Inf - Inf), which would
                // turn an Inf result into NaN.
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const uint32_t h = r[j];
                    if ((h & 0x7f800000u) != 0x7f800000u) r[j] = __float_as_uint(__uint_as_float(h) + __uint_as_float(rl[j]));
                }
                if (row_bias) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) + rbias);
                }
                const float* abase = p.aux ? p.aux + (int64_t)bidx * p.stride_aux : nullptr;
                if (vec && col0 + 32 <= p.N) {  // warp-uniform
                    // thread `lane` holds row q*32+lane: stage it ...
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        float4 v;
                        v.x = epi(__uint_as_float(r[j + 0]), cbias, col0 + j + 0, p.relu);
                        v.y = epi(__uint_as_float(r[j + 1]), cbias, col0 + j + 1, p.relu);
                        v.z = epi(__uint_as_float(r[j + 2]), cbias, col0 + j + 2, p.relu);
                        v.w = epi(__uint_as_float(r[j + 3]), cbias, col0 + j + 3, p.relu);
                        *reinterpret_cast<float4*>(stg + lane * STG_LD + j) = v;
                    }
                    __syncwarp();
                    // ... and store it back four rows x 128 bytes per instruction
#pragma unroll
                    for (int it = 0; it < 8; ++it) {
                        const int rr = it * 4 + (lane >> 3);
                        const int cc = (lane & 7) * 4;
                        float4 v = *reinterpret_cast<const float4*>(stg + rr * STG_LD + cc);
                        const int grow = m0 + q * 32 + rr;
                        if (grow < p.M) {
                            if (abase) {  // mask epilogue, read coalesced like the store
                                const float* ar = abase + (int64_t)grow * p.ld_aux + col0 + cc;
                                if (!(__ldg(ar + 0) > 0.0f)) v.x = 0.0f;
                                if (!(__ldg(ar + 1) > 0.0f)) v.y = 0.0f;
                                if (!(__ldg(ar + 2) > 0.0f)) v.z = 0.0f;
                                if (!(__ldg(ar + 3) > 0.0f)) v.w = 0.0f;
                            }
                            float* dst = cbase + (int64_t)grow * p.ldc + col0 + cc;
                            if (p.mc_store) ptx::multimem_st_v4(dst, v);
                            else *reinterpret_cast<float4*>(dst) = v;
                        }
                    }
                    __syncwarp();  // the staging tile is rewritten by the next chunk
                } else if (row_ok) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (col0 + j >= p.N) continue;
                        float v = epi(__uint_as_float(r[j]), cbias, col0 + j, p.relu);
                        if (abase && !(__ldg(abase + (int64_t)row * p.ld_aux + col0 + j) > 0.0f)) v = 0.0f;
                        if (p.mc_store) ptx::multimem_st_f32(crow + col0 + j, v);
                        else crow[col0 + j] = v;
                    }
                }
            }
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        ptx::tc_fence_after();
        ptx::tmem_dealloc<TMEM_COLS>(tmem_base);
    }
    if (threadIdx.x == 0 && *err != 0) atomicOr(p.err, *err);
}

// --------------------------------------------------------------- persistent narrow tiles
// For narrow outputs (BN = 64 / 128) with many tiles, one CTA per SM walks
// its share of the output tiles instead of one CTA per tile.  A one-tile CTA
// spends its life in two serial phases -- the TMA round trips of its few
// k-slabs, then an epilogue that stores the whole tile -- and since all CTAs
// of a wave start together, every SM loads at the same time and then stores
// at the same time (measured on 64 x [512x64].[64x512]: 2.0 + 2.2 us of load
// round trips and 3.9 us of stores per 9.3 us CTA).  Here the phases of
// consecutive tiles overlap inside the CTA:
//   warp 0      TMA producer: runs ahead through the k-slabs of all its
//               tiles, as far as the STAGES-deep ring allows;
//   warp 1      TMEM allocation + MMA issuer: two accumulator buffers (each a
//               D_hi and a D_lo of BN columns), so tile i + 1 accumulates
//               while the epilogue drains tile i;
//   warps 2-9   epilogue, two warps per TMEM lane quadrant taking alternate
//               32-column chunks: drain a buffer, release it, fused epilogue,
//               then each 32 x 32 block goes out as one TMA store from a
//               128-byte swizzled staging block (own staging area);
//   warps 10-13 split of the raw K-major A tile into hi / lo in place (split_a).
// Same arithmetic, epilogues and results as tc_gemm_kernel with one K slice.
template <int BN_, int STAGES_>
struct PCfg {
    static constexpr int BN = BN_;
    static constexpr int STAGES = STAGES_;
    static constexpr uint32_t ACC_COLS = 2 * BN_;        // D_hi | D_lo of one buffer
    static constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;  // two buffers: 256 or 512 columns
    static constexpr uint32_t A_TILE_BYTES = BM * BK * 4;
    static constexpr uint32_t B_TILE_BYTES = BN_ * BK * 4;
    static constexpr uint32_t STAGE_BYTES = 2 * A_TILE_BYTES + 2 * B_TILE_BYTES;
    static constexpr uint32_t RING_BYTES = STAGES_ * STAGE_BYTES;
    // epilogue staging: per epilogue warp two 32 x 32 fp32 blocks (4 KiB each,
    // 128-byte swizzled rows) for the TMA stores, or the STG_LD-pitched block
    // of the element-store path
    static constexpr uint32_t STG_OFF = RING_BYTES;  // a multiple of 1024
    static constexpr uint32_t STG_P_BYTES = 8 * 2 * 4096;
    static_assert(STG_P_BYTES >= STG_BYTES, "staging");
    static constexpr uint32_t BAR_OFF = STG_OFF + STG_P_BYTES;
    static constexpr uint32_t SMEM_BYTES = BAR_OFF + 512 + 1024 /*align slack*/;
    static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation is a power of two");
    static_assert(3 * STAGES_ + 5 <= 56, "barrier area");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};
constexpr int PTHREADS = 448;  // 14 warps; at most 146 registers a thread
using PCfgMid = PCfg<128, 4>;
using PCfgNarrow = PCfg<64, 6>;

// Output tile t of a one-slice GEMM: batch index and first row / column
// (grouped rasterisation in bands of 16 tile rows, as tc_gemm_kernel).
__device__ __forceinline__ void tile_coords(int t, const Params& p, int bn, int* bidx, int* m0, int* n0) {
    const int per_batch = p.tiles_m * p.tiles_n;
    const int tt = t % per_batch;
    *bidx = t / per_batch;
    constexpr int GROUP = 16;
    const int span = GROUP * p.tiles_n;
    const int g = tt / span;
    const int first_m = g * GROUP;
    const int gm = min(p.tiles_m - first_m, GROUP);
    *m0 = (first_m + (tt % span) % gm) * BM;
    *n0 = ((tt % span) / gm) * bn;
}

template <class C>
__global__ void __launch_bounds__(PTHREADS, 1)
    tc_gemm_persist_kernel(const __grid_constant__ CUtensorMap tm_a_hi, const __grid_constant__ CUtensorMap tm_a_lo,
                           const __grid_constant__ CUtensorMap tm_b_hi, const __grid_constant__ CUtensorMap tm_b_lo,
                           const __grid_constant__ CUtensorMap tm_c, const Params p) {
    constexpr int BN = C::BN;
    constexpr int STAGES = C::STAGES;
    constexpr uint32_t ACC_COLS = C::ACC_COLS, TMEM_COLS = C::TMEM_COLS;
    constexpr uint32_t A_TILE_BYTES = C::A_TILE_BYTES, B_TILE_BYTES = C::B_TILE_BYTES;
    constexpr uint32_t STAGE_BYTES = C::STAGE_BYTES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    uint64_t* empty_bar = full_bar + STAGES;
    uint64_t* conv_bar = empty_bar + STAGES;  // split_a: the stage's A tile has been split
    uint64_t* accf_bar = conv_bar + STAGES;   // [2] accumulator buffer complete (MMA -> epilogue)
    uint64_t* acce_bar = accf_bar + 2;        // [2] accumulator buffer drained (epilogue -> MMA)
    uint64_t* done_bar = acce_bar + 2;        // every MMA of this CTA has completed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
    volatile uint32_t* err = tmem_slot + 1;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int total = p.tiles_m * p.tiles_n * p.batch;
    const int num_kb = (p.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full_bar[s], 1);
            ptx::mbar_init(&empty_bar[s], 1);
            ptx::mbar_init(&conv_bar[s], 4);  // one arrival per splitting warp
        }
        for (int b = 0; b < 2; ++b) {
            ptx::mbar_init(&accf_bar[b], 1);
            ptx::mbar_init(&acce_bar[b], 8);  // one arrival per epilogue warp
        }
        ptx::mbar_init(done_bar, 1);
        *err = 0;
        ptx::fence_barrier_init();
        ptx::tma_prefetch_desc(&tm_a_hi);
        ptx::tma_prefetch_desc(&tm_a_lo);
        ptx::tma_prefetch_desc(&tm_b_hi);
        ptx::tma_prefetch_desc(&tm_b_lo);
        if (p.tma_store) ptx::tma_prefetch_desc(&tm_c);
    }
    if (warp == 1) ptx::tmem_alloc<TMEM_COLS>(tmem_slot);
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    ptx::griddep_wait();
    ptx::griddep_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ TMA producer
            uint32_t g = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                int bidx, m0, n0;
                tile_coords(t, p, BN, &bidx, &m0, &n0);
                const int za = p.a_bcast ? 0 : bidx, zb = p.b_bcast ? 0 : bidx;
                for (int kb = 0; kb < num_kb; ++kb, ++g) {
                    const int s = g % STAGES;
                    const uint32_t phase = (g / STAGES) & 1;
                    if (!ptx::mbar_wait(&empty_bar[s], phase ^ 1, err)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + s * STAGE_BYTES;
                    ptx::mbar_arrive_expect_tx(&full_bar[s], p.split_a ? STAGE_BYTES - A_TILE_BYTES : STAGE_BYTES);
                    const int kx = kb * BK;
                    ptx::tma_load_3d(st, &tm_a_hi, &full_bar[s], kx, m0, za);
                    if (!p.split_a) ptx::tma_load_3d(st + A_TILE_BYTES, &tm_a_lo, &full_bar[s], kx, m0, za);
                    ptx::tma_load_3d(st + 2 * A_TILE_BYTES, &tm_b_hi, &full_bar[s], kx, n0, zb);
                    ptx::tma_load_3d(st + 2 * A_TILE_BYTES + B_TILE_BYTES, &tm_b_lo, &full_bar[s], kx, n0, zb);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------ MMA issuer
            constexpr uint32_t idesc = ptx::idesc_tf32(BM, BN);
            uint32_t g = 0;
            bool ok = true;
            int i = 0;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++i) {
                const int buf = i & 1;
                // the epilogue has drained this buffer's previous tile
                if (!ptx::mbar_wait(&acce_bar[buf], ((i >> 1) & 1) ^ 1, err)) break;
                ptx::tc_fence_after();
                const uint32_t d_hi = tmem_base + buf * ACC_COLS, d_lo = d_hi + BN;
                for (int kb = 0; kb < num_kb; ++kb, ++g) {
                    const int s = g % STAGES;
                    const uint32_t phase = (g / STAGES) & 1;
                    if (!ptx::mbar_wait(p.split_a ? &conv_bar[s] : &full_bar[s], phase, err)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    const uint32_t st = ptx::smem_u32(smem + s * STAGE_BYTES);
                    const uint32_t a_hi = st, a_lo = st + A_TILE_BYTES;
                    const uint32_t b_hi = st + 2 * A_TILE_BYTES, b_lo = b_hi + B_TILE_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 8; ++kk) {
                        const uint32_t off = kk * 32;
                        const uint32_t acc0 = (kb | kk) != 0;
                        const uint64_t dah = ptx::smem_desc_kmajor(a_hi + off, 64);
                        const uint64_t dbh = ptx::smem_desc_kmajor(b_hi + off, 64);
                        ptx::mma_tf32(d_lo, ptx::smem_desc_kmajor(a_lo + off, 64), dbh, idesc, acc0);
                        ptx::mma_tf32(d_lo, dah, ptx::smem_desc_kmajor(b_lo + off, 64), idesc, 1);
                        ptx::mma_tf32(d_hi, dah, dbh, idesc, acc0);
                    }
                    ptx::mma_commit(&empty_bar[s]);  // slot s is free once these MMAs finish
                }
                if (ok) ptx::mma_commit(&accf_bar[buf]);
            }
            // every MMA issued here completes before the TMEM is released
            ptx::mma_commit(done_bar);
            ptx::mbar_wait(done_bar, 0, err);
        }
    } else if (warp >= 10) {
        // ---------------------------------------------------- A split (split_a)
        if (p.split_a) {
            const int ct = threadIdx.x - 320;  // 0..127
            uint32_t g = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                for (int kb = 0; kb < num_kb; ++kb, ++g) {
                    const int s = g % STAGES;
                    const uint32_t phase = (g / STAGES) & 1;
                    int okw = 0;
                    if (lane == 0) okw = ptx::mbar_wait(&full_bar[s], phase, err);
                    if (!__shfl_sync(0xffffffffu, okw, 0)) {
                        ok = false;
                        break;
                    }
                    float4* hi = reinterpret_cast<float4*>(smem + s * STAGE_BYTES);
                    float4* lo = reinterpret_cast<float4*>(smem + s * STAGE_BYTES + A_TILE_BYTES);
#pragma unroll
                    for (int k = 0; k < (int)(A_TILE_BYTES / 16) / 128; ++k) {
                        const int idx = ct + k * 128;
                        const float4 v = hi[idx];
                        float4 h, l;
                        h.x = ptx::to_tf32(v.x); l.x = ptx::to_tf32(v.x - h.x);
                        h.y = ptx::to_tf32(v.y); l.y = ptx::to_tf32(v.y - h.y);
                        h.z = ptx::to_tf32(v.z); l.z = ptx::to_tf32(v.z - h.z);
                        h.w = ptx::to_tf32(v.w); l.w = ptx::to_tf32(v.w - h.w);
                        hi[idx] = h;
                        lo[idx] = l;
                    }
                    ptx::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(&conv_bar[s]);
                }
            }
        }
    } else {
        // ---------------------------------------------------- epilogue (warps 2-9)
        const int q = warp & 3;           // TMEM lane quadrant this warp may access
        const int half = (warp - 2) >> 2;  // 0: even 32-column chunks, 1: odd
        float* stg = reinterpret_cast<float*>(smem + C::STG_OFF) + (warp - 2) * (32 * STG_LD);
        uint8_t* tstg = smem + C::STG_OFF + (warp - 2) * 2 * 4096;  // two swizzled 4 KiB blocks
        uint32_t nstore = 0;  // TMA stores issued by this warp
        const bool row_bias = p.bias_row && p.bias;
        const float* cbias = p.bias_row ? nullptr : p.bias;
        const bool vec = ((p.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
                         ((p.strideC & 3) == 0);
        int i = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++i) {
            const int buf = i & 1;
            int okw = 0;
            if (lane == 0) okw = ptx::mbar_wait(&accf_bar[buf], (i >> 1) & 1, err) && *err == 0;
            if (!__shfl_sync(0xffffffffu, okw, 0)) break;
            ptx::tc_fence_after();
            int bidx, m0, n0;
            tile_coords(t, p, BN, &bidx, &m0, &n0);
            const int row = m0 + q * 32 + lane;
            const bool row_ok = row < p.M;
            float* cbase = p.C + (int64_t)bidx * p.strideC;
            float* crow = cbase + (int64_t)row * p.ldc;
            const float rbias = (row_bias && row_ok) ? __ldg(p.bias + row) : 0.0f;
            const float* abase = p.aux ? p.aux + (int64_t)bidx * p.stride_aux : nullptr;
            const int nchunks = min(BN / 32, (p.N - n0 + 31) / 32);
            // this warp's chunks: c = half, half + 2, ...; a warp with none
            // still releases the buffer
            const int last = nchunks - 1 - ((nchunks - 1 - half) & 1);
            if (last < 0) {
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(&acce_bar[buf]);
            }
#pragma unroll 1
            for (int c = half; c < nchunks; c += 2) {
                const int col0 = n0 + c * 32;
                uint32_t r[32], rl[32];
                const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + buf * ACC_COLS + (uint32_t)(c * 32);
                ptx::tmem_ld_32x32b_x32(taddr, r);
                ptx::tmem_ld_32x32b_x32(taddr + BN, rl);
                ptx::tmem_ld_wait();
                if (c == last) {  // this warp is done with the buffer: the MMA may reuse it once all are
                    ptx::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(&acce_bar[buf]);
                }
                // a non-finite D_hi is the result (see tc_gemm_kernel)
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const uint32_t h = r[j];
                    if ((h & 0x7f800000u) != 0x7f800000u) r[j] = __float_as_uint(__uint_as_float(h) + __uint_as_float(rl[j]));
                }
                if (row_bias) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) + rbias);
                }
                if (p.tma_store) {  // warp-uniform; no mask epilogue on this path
                    // row `lane` of the block into a 128-byte swizzled staging
                    // row (16-byte chunk j at j ^ (lane & 7): conflict-free),
                    // then one TMA store of the 32 x 32 block; the box parts
                    // past M or N are not written, and a block wholly past M
                    // is not stored
                    if (m0 + q * 32 < p.M) {
                        uint8_t* blk = tstg + (nstore & 1) * 4096;
                        if (lane == 0) ptx::bulk_wait_read<1>();  // the store that used `blk` has read it
                        __syncwarp();
                        const float* cb = (cbias && col0 + 32 <= p.N) ? cbias : nullptr;  // partial chunk below
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            float4 v;
                            v.x = epi(__uint_as_float(r[4 * j + 0]), cb, col0 + 4 * j + 0, p.relu);
                            v.y = epi(__uint_as_float(r[4 * j + 1]), cb, col0 + 4 * j + 1, p.relu);
                            v.z = epi(__uint_as_float(r[4 * j + 2]), cb, col0 + 4 * j + 2, p.relu);
                            v.w = epi(__uint_as_float(r[4 * j + 3]), cb, col0 + 4 * j + 3, p.relu);
                            if (cbias && !cb) {  // last chunk of a ragged N: bias only where it exists
                                const int c4 = col0 + 4 * j;
                                v.x = c4 + 0 < p.N ? epi(__uint_as_float(r[4 * j + 0]), cbias, c4 + 0, p.relu) : 0.0f;
                                v.y = c4 + 1 < p.N ? epi(__uint_as_float(r[4 * j + 1]), cbias, c4 + 1, p.relu) : 0.0f;
                                v.z = c4 + 2 < p.N ? epi(__uint_as_float(r[4 * j + 2]), cbias, c4 + 2, p.relu) : 0.0f;
                                v.w = c4 + 3 < p.N ? epi(__uint_as_float(r[4 * j + 3]), cbias, c4 + 3, p.relu) : 0.0f;
                            }
                            *reinterpret_cast<float4*>(blk + lane * 128 + ((j ^ (lane & 7)) << 4)) = v;
                        }
                        ptx::fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            ptx::tma_store_3d(&tm_c, blk, col0, m0 + q * 32, bidx);
                            ptx::bulk_commit();
                        }
                        ++nstore;
                    }
                } else if (vec && col0 + 32 <= p.N) {  // warp-uniform
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        float4 v;
                        v.x = epi(__uint_as_float(r[j + 0]), cbias, col0 + j + 0, p.relu);
                        v.y = epi(__uint_as_float(r[j + 1]), cbias, col0 + j + 1, p.relu);
                        v.z = epi(__uint_as_float(r[j + 2]), cbias, col0 + j + 2, p.relu);
                        v.w = epi(__uint_as_float(r[j + 3]), cbias, col0 + j + 3, p.relu);
                        *reinterpret_cast<float4*>(stg + lane * STG_LD + j) = v;
                    }
                    __syncwarp();
#pragma unroll
                    for (int it = 0; it < 8; ++it) {
                        const int rr = it * 4 + (lane >> 3);
                        const int cc = (lane & 7) * 4;
                        float4 v = *reinterpret_cast<const float4*>(stg + rr * STG_LD + cc);
                        const int grow = m0 + q * 32 + rr;
                        if (grow < p.M) {
                            if (abase) {
                                const float* ar = abase + (int64_t)grow * p.ld_aux + col0 + cc;
                                if (!(__ldg(ar + 0) > 0.0f)) v.x = 0.0f;
                                if (!(__ldg(ar + 1) > 0.0f)) v.y = 0.0f;
                                if (!(__ldg(ar + 2) > 0.0f)) v.z = 0.0f;
                                if (!(__ldg(ar + 3) > 0.0f)) v.w = 0.0f;
                            }
                            *reinterpret_cast<float4*>(cbase + (int64_t)grow * p.ldc + col0 + cc) = v;
                        }
                    }
                    __syncwarp();  // the staging tile is rewritten by the next chunk
                } else if (row_ok) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (col0 + j >= p.N) continue;
                        float v = epi(__uint_as_float(r[j]), cbias, col0 + j, p.relu);
                        if (abase && !(__ldg(abase + (int64_t)row * p.ld_aux + col0 + j) > 0.0f)) v = 0.0f;
                        crow[col0 + j] = v;
                    }
                }
            }
        }
        if (lane == 0 && nstore) ptx::bulk_wait_all();  // C is written before the CTA exits
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        ptx::tc_fence_after();
        ptx::tmem_dealloc<TMEM_COLS>(tmem_base);
    }
    if (threadIdx.x == 0 && *err != 0) atomicOr(p.err, *err);
}

// --------------------------------------------------------------- split passes
// Source K-major: element (b, r, k) at src[b*sstride + r*ld + k].
template <bool VEC>
__global__ void split_rows_kernel(const float* __restrict__ src, int64_t ld, int64_t sstride, int rows, int K,
                                  int Kp, int batch, float* __restrict__ hi, float* __restrict__ lo) {
    const int kq = Kp >> 2;  // float4 groups per output row
    const int64_t total = (int64_t)batch * rows * kq;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t rr = i / kq;  // b * rows + r
        const int k = (int)(i - rr * kq) * 4;
        const int b = (int)(rr / rows);
        const int r = (int)(rr - (int64_t)b * rows);
        const float* s = src + b * sstride + r * ld;
        float v[4];
        if (VEC && k + 3 < K) {
            const float4 x = __ldg(reinterpret_cast<const float4*>(s + k));
            v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = (k + j < K) ? __ldg(s + k + j) : 0.0f;
        }
        float h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            h[j] = ptx::to_tf32(v[j]);
            l[j] = ptx::to_tf32(v[j] - h[j]);
        }
        const int64_t o = rr * Kp + k;
        *reinterpret_cast<float4*>(hi + o) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4*>(lo + o) = make_float4(l[0], l[1], l[2], l[3]);
    }
}

// Source MN-major: element (b, r, k) at src[b*sstride + k*ld + r]; transposed
// through shared memory in tiles of TR rows x TK k (32 x 128, or 64 x 64 when
// K <= 64 so that no half of the block idles on padding).  Each thread issues
// its 16 loads (32 consecutive rows per warp: 128-byte reads) before the one
// barrier, then writes 4 consecutive k of a row as float4s (a warp covers
// whole 16-byte chunks of plane rows).  The tile row pitch of TK + 1 floats
// keeps the transposing shared-memory stores conflict-free.
template <int TR, int TK>
__global__ void __launch_bounds__(256) split_transpose_kernel(const float* __restrict__ src, int64_t ld,
                                                              int64_t sstride, int rows, int K, int Kp,
                                                              float* __restrict__ hi, float* __restrict__ lo) {
    static_assert(TR * TK == 4096, "16 elements per thread");
    constexpr int KT = 256 / TR;  // load phase: threads along k per pass
    constexpr int CK = TK / 4;    // store phase: float4 chunks per tile row
    constexpr int RP = 256 / CK;  // store phase: rows per pass
    __shared__ float tile[TR][TK + 1];  // [row][k]
    const int b = blockIdx.z;
    const int r0 = blockIdx.x * TR;
    const int k0 = blockIdx.y * TK;
    const float* s = src + b * sstride;
    const int tx = threadIdx.x % TR, ty = threadIdx.x / TR;  // load phase: row fastest
    float v[TK / KT];
#pragma unroll
    for (int i = 0; i < TK / KT; ++i) {
        const int k = k0 + ty + KT * i;
        const int r = r0 + tx;
        v[i] = (k < K && r < rows) ? __ldg(s + (int64_t)k * ld + r) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < TK / KT; ++i) tile[tx][ty + KT * i] = v[i];
    __syncthreads();
    const int c = threadIdx.x % CK, rr = threadIdx.x / CK;
#pragma unroll
    for (int pass = 0; pass < TR / RP; ++pass) {
        const int rl = rr + RP * pass;
        const int r = r0 + rl;
        const int k = k0 + 4 * c;
        if (r >= rows || k >= Kp) continue;
        float h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float x = tile[rl][4 * c + j];
            h[j] = ptx::to_tf32(x);
            l[j] = ptx::to_tf32(x - h[j]);
        }
        const int64_t o = ((int64_t)b * rows + r) * Kp + k;  // Kp % 4 == 0, k % 4 == 0: 16-byte aligned
        *reinterpret_cast<float4*>(hi + o) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4*>(lo + o) = make_float4(l[0], l[1], l[2], l[3]);
    }
}

// --------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 3-D map over a K-major plane [batch][rows][Kp] with box {BK, box_rows, 1}.
static bool make_plane_map(CUtensorMap* m, const float* base, int K, int rows, int batch, int Kp, int box_rows) {
    auto enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)batch};
    cuuint64_t strides[2] = {(cuuint64_t)Kp * 4, (cuuint64_t)Kp * 4 * (cuuint64_t)rows};
    cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 3-D map over a raw K-major fp32 operand [batch][rows][K] (row stride ld,
// batch stride bstride, elements): the tensor-core kernel splits its tiles in
// shared memory.  Same box and swizzle as the planes.
static bool make_raw_map(CUtensorMap* m, const float* base, int K, int rows, int batch, int64_t ld, int64_t bstride,
                         int box_rows) {
    auto enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)batch};
    const int64_t bs = batch > 1 ? bstride : ld * rows;
    cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)bs * 4};
    cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 3-D map over C [batch][M][ldc] for TMA stores of 32 x 32 blocks (128-byte
// swizzled rows in shared memory).  False when C's base or strides are not
// 16-byte multiples.
static bool make_c_map(CUtensorMap* m, float* C, int M, int N, int batch, int64_t ldc, int64_t strideC) {
    if ((reinterpret_cast<uintptr_t>(C) & 15) || (ldc & 3) || (batch > 1 && (strideC & 3))) return false;
    auto enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)batch};
    const int64_t bs = batch > 1 ? strideC : ldc * M;
    cuuint64_t strides[2] = {(cuuint64_t)ldc * 4, (cuuint64_t)bs * 4};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, C, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

static int launch_split(const float* src, bool kmajor, int64_t ld, int64_t sstride, int rows, int K, int Kp,
                        int batch, float* hi, float* lo, cudaStream_t s) {
    if (rows == 0 || Kp == 0) return JST_OK;
    if (kmajor) {
        const bool vec = ((ld & 3) == 0) && ((sstride & 3) == 0) && ((reinterpret_cast<uintptr_t>(src) & 15) == 0);
        const int64_t total = (int64_t)batch * rows * (Kp / 4);
        const int threads = 256;
        const int64_t want = (total + threads - 1) / threads;
        const int blocks = (int)(want < 148 * 16 ? want : 148 * 16);
        ProfScope prof(s, KID_SPLIT_ROWS);
        if (vec)
            split_rows_kernel<true><<<blocks, threads, 0, s>>>(src, ld, sstride, rows, K, Kp, batch, hi, lo);
        else
            split_rows_kernel<false><<<blocks, threads, 0, s>>>(src, ld, sstride, rows, K, Kp, batch, hi, lo);
    } else if (Kp <= 64) {
        dim3 grid((rows + 63) / 64, 1, batch);
        ProfScope prof(s, KID_SPLIT_TRANSPOSE);
        split_transpose_kernel<64, 64><<<grid, 256, 0, s>>>(src, ld, sstride, rows, K, Kp, hi, lo);
    } else {
        dim3 grid((rows + 31) / 32, (Kp + 127) / 128, batch);
        ProfScope prof(s, KID_SPLIT_TRANSPOSE);
        split_transpose_kernel<32, 128><<<grid, 256, 0, s>>>(src, ld, sstride, rows, K, Kp, hi, lo);
    }
    return cudaPeekAtLastError() == cudaSuccess ? JST_OK : JST_ERR_CUDA;
}

}  // namespace tc

// Tile configuration of a GEMM: narrow tiles for narrow outputs, and for short
// K (the output then dominates and two co-resident CTAs overlap one's
// epilogue with the other's main loop); the 256-wide tile otherwise.
int tc_pick_bn(int M, int N, int K) {
    (void)M;
    if (N <= 64) return 64;
    if (N <= 128 || K <= 256) return 128;
    return 256;
}

// Split K when the output tiles fill less than half a wave (148 one-CTA or
// 296 two-CTA slots): as many slices as still fit in the wave, each at least
// 64 BK steps (K = 1024) long, at most 16.  The count is normalised so that
// no slice is empty.
int tc_split_k(const GemmArgs& a) {
    const int bn = tc_pick_bn(a.M, a.N, a.K);
    const int64_t slots = bn == 256 ? 148 : 296;
    const int64_t tiles = (int64_t)((a.M + tc::BM - 1) / tc::BM) * ((a.N + bn - 1) / bn) * a.batch;
    const int num_kb = (a.K + tc::BK - 1) / tc::BK;
    if (tiles <= 0 || tiles >= slots / 2) return 1;
    int S = (int)std::min<int64_t>(std::min<int64_t>(slots / tiles, num_kb / 64), 16);
    if (S <= 1) return 1;
    const int per = (num_kb + S - 1) / S;
    return (num_kb + per - 1) / per;
}

// Planes of the operands that vary over the batch; a broadcast (stride 0)
// operand is split once.  Then the split-K partials, if any.
static bool a_broadcast(const GemmArgs& a) { return a.batch > 1 && a.strideA == 0; }
static bool b_broadcast(const GemmArgs& a) { return a.batch > 1 && a.strideB == 0; }

// Split A inside the kernel (no A planes) when the tile is narrow -- the GEMM
// then streams A once from memory instead of reading it, writing two planes
// and reading those back -- and A is K-major with TMA-compatible strides.
// The 256-wide configuration keeps the split pass: there the MMA loop is
// already bounded by shared-memory bandwidth.
static bool use_split_a(const GemmArgs& a) {
    if (a.transA || tc_pick_bn(a.M, a.N, a.K) == 256) return false;
    if ((reinterpret_cast<uintptr_t>(a.A) & 15) || (a.lda & 3)) return false;
    if (a.batch > 1 && !a_broadcast(a) && (a.strideA & 3)) return false;
    return true;
}

size_t tc_workspace_bytes(const GemmArgs& a) {
    const size_t Kp = (size_t)((a.K + 3) & ~3);
    const size_t ab = use_split_a(a) ? 0 : (a_broadcast(a) ? 1 : (size_t)a.batch);
    const size_t bb = b_broadcast(a) ? 1 : (size_t)a.batch;
    const int S = tc_split_k(a);
    const size_t part = S > 1 ? (size_t)S * a.batch * a.M * a.N : 0;
    return (2 * Kp * ((size_t)a.M * ab + (size_t)a.N * bb) + part) * sizeof(float);
}

int tc_split(const float* src, int kmajor, int64_t ld, int64_t sstride, int rows, int K, int batch, float* hi,
             float* lo, cudaStream_t s) {
    const int rc = tc::launch_split(src, kmajor != 0, ld, sstride, rows, K, (K + 3) & ~3, batch, hi, lo, s);
    return rc ? set_status(rc, "split pass failed to launch") : JST_OK;
}

// Launch one configuration; its shared-memory opt-in is set once per device.
template <class Cf>
static int launch_cfg(const CUtensorMap& a_hi, const CUtensorMap& a_lo, const CUtensorMap& b_hi,
                      const CUtensorMap& b_lo, const tc::Params& p, unsigned grid, cudaStream_t s, bool pdl) {
    static bool attr_set[64] = {};
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lk(mu);
        if (dev >= 0 && dev < 64 && !attr_set[dev]) {
            if (cudaFuncSetAttribute(tc::tc_gemm_kernel<Cf>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Cf::SMEM_BYTES) != cudaSuccess)
                return set_status(JST_ERR_CUDA, "cudaFuncSetAttribute(tc_gemm_kernel) failed");
            attr_set[dev] = true;
        }
    }
    {
        ProfScope prof(s, KID_TC_GEMM);
        if (pdl) {
            if (launch_dependent(tc::tc_gemm_kernel<Cf>, dim3(grid), dim3(tc::THREADS), Cf::SMEM_BYTES, s, a_hi, a_lo,
                                 b_hi, b_lo, p) != cudaSuccess)
                return set_status(JST_ERR_CUDA, "tc_gemm_kernel launch failed");
        } else {
            tc::tc_gemm_kernel<Cf><<<grid, tc::THREADS, Cf::SMEM_BYTES, s>>>(a_hi, a_lo, b_hi, b_lo, p);
        }
    }
    if (cudaPeekAtLastError() != cudaSuccess) return set_status(JST_ERR_CUDA, "tc_gemm_kernel launch failed");
    return JST_OK;
}

// Launch the persistent narrow-tile kernel on `grid` CTAs (one per SM).
template <class Cf>
static int launch_persist(const CUtensorMap& a_hi, const CUtensorMap& a_lo, const CUtensorMap& b_hi,
                          const CUtensorMap& b_lo, const CUtensorMap& c_map, const tc::Params& p, unsigned grid,
                          cudaStream_t s, bool pdl) {
    static bool attr_set[64] = {};
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lk(mu);
        if (dev >= 0 && dev < 64 && !attr_set[dev]) {
            if (cudaFuncSetAttribute(tc::tc_gemm_persist_kernel<Cf>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Cf::SMEM_BYTES) != cudaSuccess)
                return set_status(JST_ERR_CUDA, "cudaFuncSetAttribute(tc_gemm_persist_kernel) failed");
            attr_set[dev] = true;
        }
    }
    {
        ProfScope prof(s, KID_TC_GEMM);
        if (pdl) {
            if (launch_dependent(tc::tc_gemm_persist_kernel<Cf>, dim3(grid), dim3(tc::PTHREADS), Cf::SMEM_BYTES, s,
                                 a_hi, a_lo, b_hi, b_lo, c_map, p) != cudaSuccess)
                return set_status(JST_ERR_CUDA, "tc_gemm_persist_kernel launch failed");
        } else {
            tc::tc_gemm_persist_kernel<Cf><<<grid, tc::PTHREADS, Cf::SMEM_BYTES, s>>>(a_hi, a_lo, b_hi, b_lo, c_map,
                                                                                      p);
        }
    }
    if (cudaPeekAtLastError() != cudaSuccess) return set_status(JST_ERR_CUDA, "tc_gemm_persist_kernel launch failed");
    return JST_OK;
}

// SMs of the current device (the persistent kernel's grid).
static int sm_count() {
    static std::atomic<int> cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return 148;
    }
    int n = cached[dev].load(std::memory_order_relaxed);
    if (!n) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = 148;
        }
        cached[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

// Narrow tiles (64 / 128 columns) in one K slice, written straight to C, and
// at least two tiles per SM: the persistent kernel overlaps each tile's
// epilogue with the next tile's loads and MMAs.  With fewer tiles a CTA per
// tile spreads the work over more SMs (64 x [512x512].[512x64]: 256 tiles of
// 32 k-slabs ran 31 us one per CTA, 43 us two per persistent CTA).
static bool use_persistent(int bn, int64_t tiles, int kslices, int mc_store) {
    return kslices == 1 && !mc_store && bn <= 128 && tiles >= 2LL * sm_count();
}

int tc_gemm_planes(const float* a_hi, const float* a_lo, const float* b_hi, const float* b_lo, int M, int N, int K,
                   int batch, float* C, int64_t ldc, int64_t strideC, const float* bias, int relu, uint32_t* err,
                   cudaStream_t s, int mc_store, const float* aux, int64_t ld_aux, int64_t stride_aux, int bias_row,
                   int a_bcast, int b_bcast, int kslices, int split_a, int64_t lda_raw, int64_t strideA_raw,
                   int pdl) {
    using namespace tc;
    const int Kp = (K + 3) & ~3;
    const int num_kb = (K + BK - 1) / BK;
    if (kslices < 1 || kslices > num_kb) return set_status(JST_ERR_ARG, "tc: bad split-K slice count");
    const int kb_per_slice = (num_kb + kslices - 1) / kslices;
    if ((num_kb + kb_per_slice - 1) / kb_per_slice != kslices)  // a slice would be empty
        return set_status(JST_ERR_ARG, "tc: split-K slice count leaves a slice empty");
    const int ab = a_bcast ? 1 : batch, bb = b_bcast ? 1 : batch;
    const int bn = tc_pick_bn(M, N, K);
    if (split_a && bn == 256) return set_status(JST_ERR_ARG, "tc: in-kernel A split needs a narrow tile");
    CUtensorMap m_ahi, m_alo, m_bhi, m_blo;
    const bool a_ok = split_a ? make_raw_map(&m_ahi, a_hi, K, M, ab, lda_raw, strideA_raw, BM)
                              : (make_plane_map(&m_ahi, a_hi, K, M, ab, Kp, BM) &&
                                 make_plane_map(&m_alo, a_lo, K, M, ab, Kp, BM));
    if (split_a) m_alo = m_ahi;  // not read
    if (!a_ok || !make_plane_map(&m_bhi, b_hi, K, N, bb, Kp, bn) || !make_plane_map(&m_blo, b_lo, K, N, bb, Kp, bn))
        return set_status(JST_ERR_CUDA, "cuTensorMapEncodeTiled failed");
    Params p;
    p.M = M; p.N = N; p.K = K; p.batch = batch;
    p.C = C; p.ldc = ldc; p.strideC = strideC;
    p.bias = bias; p.bias_row = bias_row; p.relu = relu;
    p.tiles_m = (M + BM - 1) / BM;
    p.tiles_n = (N + bn - 1) / bn;
    p.err = err;
    p.mc_store = mc_store;
    p.aux = aux;
    p.ld_aux = ld_aux;
    p.stride_aux = stride_aux;
    p.a_bcast = a_bcast;
    p.b_bcast = b_bcast;
    p.kslices = kslices;
    p.kb_per_slice = kb_per_slice;
    p.split_a = split_a;
    p.tma_store = 0;
    const int64_t grid = (int64_t)p.tiles_m * p.tiles_n * batch * kslices;
    if (grid > 0x7fffffff) return set_status(JST_ERR_ARG, "tc: too many tiles");
    int rc;
    if (use_persistent(bn, grid, kslices, mc_store)) {
        // C through TMA stores when its layout allows them (16-byte aligned
        // base and strides) and no mask is read; element stores otherwise
        CUtensorMap m_c = m_ahi;  // not read unless tma_store
        p.tma_store = !aux && make_c_map(&m_c, C, M, N, batch, ldc, strideC) ? 1 : 0;
        const unsigned pgrid = (unsigned)std::min<int64_t>(grid, sm_count());
        if (bn == 128) rc = launch_persist<PCfgMid>(m_ahi, m_alo, m_bhi, m_blo, m_c, p, pgrid, s, pdl != 0);
        else rc = launch_persist<PCfgNarrow>(m_ahi, m_alo, m_bhi, m_blo, m_c, p, pgrid, s, pdl != 0);
        return rc;
    }
    if (bn == 256) rc = launch_cfg<CfgWide>(m_ahi, m_alo, m_bhi, m_blo, p, (unsigned)grid, s, pdl != 0);
    else if (bn == 128) rc = launch_cfg<CfgMid>(m_ahi, m_alo, m_bhi, m_blo, p, (unsigned)grid, s, pdl != 0);
    else rc = launch_cfg<CfgNarrow>(m_ahi, m_alo, m_bhi, m_blo, p, (unsigned)grid, s, pdl != 0);
    return rc;
}

// Split both operands into `workspace` and run the tensor-core kernel;
// `err` receives the kernel's timeout flag.
static int tc_gemm_launch(const GemmArgs& a, void* workspace, uint32_t* err, cudaStream_t s) {
    const int Kp = (a.K + 3) & ~3;
    float* ws = static_cast<float*>(workspace);
    const bool abc = a_broadcast(a), bbc = b_broadcast(a), sa = use_split_a(a);
    const int ab = abc ? 1 : a.batch, bb = bbc ? 1 : a.batch;
    const size_t a_plane = sa ? 0 : (size_t)ab * a.M * Kp;
    const size_t b_plane = (size_t)bb * a.N * Kp;
    float* a_hi = ws;
    float* a_lo = a_hi + a_plane;
    float* b_hi = a_lo + a_plane;
    float* b_lo = b_hi + b_plane;
    float* part = b_lo + b_plane;
    // op(A) rows are M: K-major unless A is stored transposed.
    int rc = sa ? JST_OK : tc_split(a.A, !a.transA, a.lda, a.strideA, a.M, a.K, ab, a_hi, a_lo, s);
    if (rc) return rc;
    const float* ah = sa ? a.A : a_hi;
    // op(B)^T rows are N: K-major when B is stored [N, K] (transB).
    rc = tc_split(a.B, a.transB, a.ldb, a.strideB, a.N, a.K, bb, b_hi, b_lo, s);
    if (rc) return rc;
    // the GEMM follows the B split on `s`: launched as its programmatic
    // dependent, its set-up overlaps the split's tail
    const int S = tc_split_k(a);
    if (S <= 1)
        return tc_gemm_planes(ah, a_lo, b_hi, b_lo, a.M, a.N, a.K, a.batch, a.C, a.ldc, a.strideC, a.bias, a.relu, err,
                              s, 0, a.aux, a.ld_aux, a.stride_aux, a.bias_row, abc, bbc, 1, sa, a.lda, a.strideA,
                              /*pdl=*/1);
    rc = tc_gemm_planes(ah, a_lo, b_hi, b_lo, a.M, a.N, a.K, a.batch, part, a.N, (int64_t)a.M * a.N, nullptr, 0, err,
                        s, 0, nullptr, 0, 0, 0, abc, bbc, S, sa, a.lda, a.strideA, /*pdl=*/1);
    if (rc) return rc;
    return splitk_reduce_run(splitk_reduce_args(a, part, S), s);
}

int tc_gemm_run(const GemmArgs& a, void* workspace, cudaStream_t s) {
    return tc_gemm_launch(a, workspace, device_error_word(), s);
}

// ----------------------------------------------------------------------------
// Allocation-free variant (jst_gemm_tc_noalloc).
//
// Some callers cannot call cudaMalloc: hosts whose device memory is owned by
// another allocator that forbids side allocations (an embedding runtime that
// hands the library a fixed arena), embedders that must size all device
// memory up front, and latency-critical code that cannot afford cudaMalloc /
// cudaFree, which may synchronise the whole device.  For them the split
// planes (and split-K partials) of the 3xTF32 kernel live in this fixed,
// file-scope device array instead of a workspace from the library's pool.
//
// The array is NOALLOC_SCRATCH_BYTES (64 MiB) and belongs to this module: the
// CUDA runtime reserves it on a device when the module is loaded there (on
// first use with lazy module loading, which is the default; at context
// creation with CUDA_MODULE_LOADING=EAGER), and it is held until the process
// exits.  The real limit is what tc_workspace_bytes() returns for the request:
//   2 * Kp * (M * Ba + N * Bb) * 4 bytes of hi / lo planes (Kp = K rounded up
//   to 4; Ba, Bb = batch, or 1 for an operand with batch stride 0; Ba = 0
//   when A is split inside the kernel, which narrow tiles of a K-major A do)
//   + S * batch * M * N * 4 bytes of split-K partials (S > 1 only when the
//   output tiles fill less than half the SMs).
// A request above 64 MiB is rejected with JST_ERR_ARG before any device work.
//
// The array is shared by every call on a device and keeps the previous call's
// planes.  Nothing in it has to start at zero: the split kernels rewrite every
// row and every padded column of the planes a call uses, and every split-K
// partial is written before the reduce reads it.  Two calls whose work
// overlaps on the GPU (on different streams, or from different threads) race
// on the array and give wrong results: serialise them.
//
// The kernel's timeout word is file-scope too.  It starts at zero when the
// module loads, a kernel whose bounded wait gave up ORs its flag into it, and
// jst_device_error() reads and clears it together with the word of the
// allocating entry points -- so a timed-out call is reported the same way on
// both paths.  The device addresses of both arrays are looked up once per
// device and cached; cudaDeviceReset() (which unloads the module) is not
// supported in a process that has called this entry point.
// ----------------------------------------------------------------------------
constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(64) << 20;
static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_SCRATCH_BYTES / sizeof(float)];
static __device__ __align__(256) uint32_t g_noalloc_err;

namespace {
struct NoAllocDevice {
    bool ready = false;
    float* scratch = nullptr;  // device address of g_noalloc_scratch on this device
    uint32_t* err = nullptr;   // device address of g_noalloc_err on this device
};
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[64];

// Once per device, with that device current: resolve the device addresses of
// the file-scope arrays.  Their host-side names are only stand-ins and must
// never be passed to a kernel.
int noalloc_setup(int dev, NoAllocDevice** out) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoAllocDevice& d = g_noalloc_dev[dev];
    if (!d.ready) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return set_status(JST_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed");
        }
        d.scratch = static_cast<float*>(p);
        e = cudaGetSymbolAddress(&p, g_noalloc_err);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return set_status(JST_ERR_CUDA, "cudaGetSymbolAddress(error word) failed");
        }
        d.err = static_cast<uint32_t*>(p);
        d.ready = true;
    }
    *out = &d;
    return JST_OK;
}
}  // namespace

// The noalloc timeout word of device `dev`: *out = its value (0 when the
// entry point never ran there), then cleared.  Called by jst_device_error()
// after it has synchronised the device.
int noalloc_take_error(int dev, uint32_t* out) {
    *out = 0;
    if (dev < 0 || dev >= 64) return JST_OK;
    uint32_t* w = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (g_noalloc_dev[dev].ready) w = g_noalloc_dev[dev].err;
    }
    if (!w) return JST_OK;
    if (cudaMemcpy(out, w, sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return set_status(JST_ERR_CUDA, "reading the scratch error word failed");
    }
    if (*out && cudaMemset(w, 0, sizeof(uint32_t)) != cudaSuccess) {
        cudaGetLastError();
        return set_status(JST_ERR_CUDA, "clearing the scratch error word failed");
    }
    return JST_OK;
}

// Host-side stand-in for a timed-out noalloc kernel (jst_test_set_device_error).
int noalloc_set_error(int dev, uint32_t value) {
    NoAllocDevice* nd = nullptr;
    int rc = noalloc_setup(dev, &nd);
    if (rc) return rc;
    if (cudaMemcpy(nd->err, &value, sizeof(value), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaGetLastError();
        return set_status(JST_ERR_CUDA, "writing the scratch error word failed");
    }
    return JST_OK;
}

}  // namespace jst

extern "C" int jst_gemm_tc_noalloc(const jst_gemm_desc* d) {
    using namespace jst;
    GemmArgs a{};
    int rc = validate_gemm_desc(d, &a);
    if (rc) return rc;
    if (d->kernel != JST_KERNEL_AUTO && d->kernel != JST_KERNEL_TC3XTF32)
        return set_status(JST_ERR_ARG, "jst_gemm_tc_noalloc runs the tensor-core kernel only");
    int dev = -1, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
        cudaGetLastError();
        return set_status(JST_ERR_NO_DEVICE, "no CUDA device available");
    }
    if (major != 10) return set_status(JST_ERR_NO_DEVICE, "libjstorch_gemm is built for sm_100a (B200) only");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(d->stream);
    if (a.M == 0 || a.N == 0) return set_status(JST_OK, nullptr);
    if (a.K == 0) {
        rc = fill_epilogue_run(a, s);
        return rc ? rc : set_status(JST_OK, nullptr);
    }
    const size_t need = tc_workspace_bytes(a);
    if (need > NOALLOC_SCRATCH_BYTES) {
        char msg[160];
        std::snprintf(msg, sizeof(msg),
                      "jst_gemm_tc_noalloc: split planes need %zu bytes, above the fixed %zu-byte scratch", need,
                      NOALLOC_SCRATCH_BYTES);
        return set_status(JST_ERR_ARG, msg);
    }
    NoAllocDevice* nd = nullptr;
    rc = noalloc_setup(dev, &nd);
    if (rc) return rc;
    // the timeout word is not cleared here: a flag left by an earlier call
    // stays set until jst_device_error() reads it
    rc = tc_gemm_launch(a, nd->scratch, nd->err, s);
    return rc ? rc : set_status(JST_OK, nullptr);
}
