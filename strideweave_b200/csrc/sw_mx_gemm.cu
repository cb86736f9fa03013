// sw_mx_gemm.cu - block-scaled MX contraction on the 5th-generation tensor
// cores: C[m, n] = sum_k A[m, k] * B[n, k] with E4M3 (kind::mxf8f6f4) or
// packed E2M1 (kind::mxf4) payloads and E8M0 per-32 scales, fp32 accumulated
// in TMEM.
//
// One persistent CTA per SM walks 128 x BN output tiles.  Warp roles:
//   warp 0 - TMA producer: 2-D tiled loads of the payload tiles (128-byte
//            swizzled rows) and 1-D bulk loads of the scale atoms into a
//            3- or 4-stage shared-memory ring;
//   warp 1 - allocates TMEM; one thread copies each stage's scale atoms from
//            shared memory into TMEM (tcgen05.cp .32x128b.warpx4) and issues
//            the tcgen05.mma block_scale instructions, committing each stage
//            back to the producer and each finished tile to the epilogue;
//   warps 2.. - epilogue: tcgen05.ld of the accumulator.  Results with a unit
//            pitch are staged in shared memory and written by TMA bulk stores
//            by eight warps, two per TMEM sub-partition, each holding half of
//            the tile's columns in registers: the accumulator is released as
//            soon as it is read, so the stores overlap the next tile's MMAs
//            (3-stage ring).  Other results are stored from registers by four
//            warps.
// The scale atoms are read exactly as the carrier stores them (the
// SW_SCALES_TC128 placement): a 512-byte atom holds 128 rows x 4 blocks in the
// order the tcgen05.cp replication expects, so no shuffle is needed.
//
// Every mbarrier wait is bounded; a wait that gives up records SW_ERR_TIMEOUT
// and its role unwinds, waiting (bounded) for its own copies and MMAs in
// flight before the CTA frees TMEM and exits.
//
// Reference counterpart: CpuMatmulOperation::_forward
// (src/strideweave/carriers/cpu/native/ops/matmul.cpp:45-113) contracts mode 1
// of both operands, i.e. C = A * B^T with both operands K-major, as here.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "sw_common.cuh"
#include "sw_ptx.cuh"
#include "sw_tma.cuh"

namespace sw {
namespace {

#ifndef SW_GEMM_RASTER_GROUP_E4M3
#define SW_GEMM_RASTER_GROUP_E4M3 16  // M blocks per raster group (measured, below)
#endif
#ifndef SW_GEMM_RASTER_GROUP_E2M1
#define SW_GEMM_RASTER_GROUP_E2M1 8
#endif
constexpr int kBM = 128;
constexpr int kBKBytes = 128;  // payload bytes of K per stage (one 128B swizzle row)
constexpr int kTmemCols = 512;

// Epilogues.  kEpiDirect stores from registers (any pitches, accumulation into
// C).  The staged ones drain the accumulator into shared memory and write it
// with TMA bulk stores that run while the next tile's MMAs do; the TMEM
// accumulator is released as soon as it is read:
//   kEpiBf16Rows - bf16, row-major C, the whole 128 x BN tile staged with the
//                  128-byte swizzle;
//   kEpiF32Rows  - fp32, row-major C, 128 x 32 chunks (128-byte swizzle)
//                  rotating through kOutBufs buffers;
//   kEpiF32Cols  - fp32, column-major C, the same chunks stored [32 n][128 m].
// In the staged epilogues warp w drains TMEM sub-partition w % 4 (rows
// 32 (w % 4) ..) and column half (w - 2) / 4; each half has its own share of
// the staging memory, named barrier and store-issuing thread.
constexpr int kEpiDirect = 0;
constexpr int kEpiBf16Rows = 1;
constexpr int kEpiF32Rows = 2;
constexpr int kEpiF32Cols = 3;
constexpr int kOutBufs = 4;
constexpr int kChunkBytes = kBM * 32 * 4;  // one 128 x 32 fp32 chunk
constexpr int kMaxRouted = 8;              // destinations of a routed contraction (ranks of a node)

// Where a routed contraction writes: row block q at dest[q] (see GemmArgs).
struct Route {
    int count;
    int64_t rows_per_dest;
    float* dest[kMaxRouted];
    int first;  // the destination whose row block the walk starts with
};

template <int FMT, int BN, int kStages, int kEpi>
struct Cfg {
    static constexpr int kEpiWarps = kEpi == kEpiDirect ? 4 : 8;
    static constexpr int kEpiThreads = 32 * kEpiWarps;
    static constexpr int kThreads = 64 + kEpiThreads;             // producer + MMA warps + epilogue
    static constexpr int kAtoms = FMT == SW_MX_E4M3 ? 1 : 2;      // scale atoms (4 blocks) per stage
    static constexpr int kABytes = kBM * kBKBytes;                 // 16 KiB
    static constexpr int kBBytes = BN * kBKBytes;
    static constexpr int kSfaBytes = kAtoms * 512;
    static constexpr int kSfbBytes = (BN / 128) * kAtoms * 512;
    static constexpr int kMmaPerStage = 4;                         // K=32 (E4M3) or K=64 (E2M1) each
    static constexpr int kSfaCols = 4 * kAtoms;
    static constexpr int kSfbCols = 4 * kAtoms * (BN / 128);
    static constexpr int kSfColsPerStage = kSfaCols + kSfbCols;
    static constexpr int kAccCol = 0;
    static constexpr int kSfCol0 = BN;                             // scale columns follow the accumulator
    static_assert(BN + kStages * kSfColsPerStage <= kTmemCols, "TMEM budget");
    static_assert(kEpi == kEpiDirect || BN == 256, "the staged epilogues split a 256-column tile in two halves");
    static constexpr int kOffA = 0;
    static constexpr int kOffB = kOffA + kStages * kABytes;
    static constexpr int kOffSfa = kOffB + kStages * kBBytes;
    static constexpr int kOffSfb = kOffSfa + kStages * kSfaBytes;
    static constexpr int kOffBar = kOffSfb + kStages * kSfbBytes;
    static constexpr int kNumBars = 2 * kStages + 3;
    static constexpr int kOffSlot = kOffBar + kNumBars * 8;
    static constexpr int kStageOutBytes =
        kEpi == kEpiBf16Rows ? kBM * BN * 2 : (kEpi == kEpiDirect ? 0 : kOutBufs * kChunkBytes);
    static constexpr int kOffOut = (kOffSlot + 16 + 1023) / 1024 * 1024;
    static constexpr int kSmemBytes = kOffOut + kStageOutBytes + 1024;  // + alignment slack
    static_assert(kSmemBytes <= 232448, "shared memory budget");
    static constexpr uint32_t kStageTx = kABytes + kBBytes + kSfaBytes + kSfbBytes;
};

// A count known at compile time, passed where a runtime int also fits (the
// full stages of the MMA issue loop unroll with it as a constant).
template <int V>
struct Count {
    __device__ constexpr operator int() const { return V; }
};

// Instruction descriptor of a block-scaled MMA (E8M0 scales, K-major A and B).
__device__ __forceinline__ uint32_t make_idesc(uint32_t fmt_code, int M, int N, uint32_t sfa_id, uint32_t sfb_id) {
    return (sfb_id << 4) | (fmt_code << 7) | (fmt_code << 10) | (uint32_t(N >> 3) << 17) | (1u << 23) |
           (uint32_t(M >> 4) << 24) | (sfa_id << 29);
}

struct GemmArgs {
    const uint8_t* sfa;
    const uint8_t* sfb;
    void* c;
    int64_t ldc_m, ldc_n;
    int M, N, K;          // K in elements
    int k_stages;         // ceil(payload row bytes / 128): the last stage may be partly past K
    int katoms;           // scale atoms per row group (ceil(K/128))
    int row_bytes;        // payload bytes of one operand row (K or K/2)
    int b_groups;         // 128-row groups in B's scale plane (ceil(batch N / 128))
    int ragged_k;         // the last stage holds fewer than kAtoms atoms or kMmaPerStage MMAs
    int last_atoms;       // scale atoms of the last stage
    int last_mmas;        // MMAs of the last stage (32 payload bytes each)
    int beta_one;
    int out_bf16;
    int batch;            // stacked problems (block-diagonal), 1 for one contraction
    int64_t c_batch;      // elements between consecutive problems' C (direct epilogue)
    // routed results (Float32; staged rows epilogue, or the direct one for
    // narrow N): C rows [q rows_per_dest, (q + 1) rows_per_dest) go to
    // dest[q], row-major with pitch ldc_m
    int routed;
    int64_t rows_per_dest;
    float* dest[kMaxRouted];
    // Row tiles the walk is rotated by (0 <= rotate_m < tiles along M): tile
    // row mb is computed where mb - rotate_m (mod the tile rows) would be.
    // Ranks of a routed K-split each start at a different owner's block, so
    // at any moment every owner receives from one writer, not from all.
    int rotate_m;
};

template <int FMT, int BN, int kStages, int kEpi>
__global__ void __launch_bounds__(kEpi == kEpiDirect ? 192 : 320, 1)
    mx_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_c, const GemmArgs args) {
    using C = Cfg<FMT, BN, kStages, kEpi>;
    static_assert(C::kThreads == (kEpi == kEpiDirect ? 192 : 320), "launch bounds");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = ptx::smem_addr(smem);
    const uint32_t bar_full = sbase + C::kOffBar;             // kStages barriers
    const uint32_t bar_empty = bar_full + kStages * 8;        // kStages barriers
    const uint32_t bar_tmem_full = bar_empty + kStages * 8;
    const uint32_t bar_tmem_empty = bar_tmem_full + 8;
    const uint32_t bar_drain = bar_tmem_empty + 8;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffSlot);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            ptx::mbar_init(bar_full + 8 * s, 1);
            ptx::mbar_init(bar_empty + 8 * s, 1);
        }
        ptx::mbar_init(bar_tmem_full, 1);
        ptx::mbar_init(bar_tmem_empty, C::kEpiThreads);
        ptx::mbar_init(bar_drain, 1);
        ptx::fence_barrier_init();
        ptx::prefetch_tmap(&tmap_a);
        ptx::prefetch_tmap(&tmap_b);
        if (kEpi != kEpiDirect) ptx::prefetch_tmap(&tmap_c);
    }
    if (warp == 1) {
        ptx::tmem_alloc(ptx::smem_addr(tmem_slot), kTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // barrier set-up, descriptor prefetch and the TMEM allocation overlap the
    // previous grid's tail; operands are read only after it completes
    pdl_enter();

    // ragged extents: the last tile row / column reaches past M / N; its
    // operand rows there are zero-filled by TMA and its results are not stored
    const int num_m = (args.M + kBM - 1) / kBM;
    const int num_n = (args.N + BN - 1) / BN;
    const int per_batch = num_m * num_n;
    const int num_tiles = args.batch * per_batch;
    // M blocks per raster group: the tiles of a group share B's panels in L2,
    // so B crosses HBM once per group.  MXFP8 at 65536 x 16384 x 16384 back to
    // back under the power cap, groups of 4 / 8 / 16 / 32: 1.80 / 1.90 / 1.95 /
    // 1.93 PF/s (SM clock 1354 / 1372-1414 / 1436-1440 / 1425 MHz; fewer HBM
    // bytes leave more of the power budget to the tensor cores); at 8192^3,
    // 16 against 8: MXFP8 2.30 against 2.24 PF/s, MXFP4 4.27 against 4.39.
    constexpr int kGroup = FMT == SW_MX_E4M3 ? SW_GEMM_RASTER_GROUP_E4M3 : SW_GEMM_RASTER_GROUP_E2M1;

    // Tile t of a batched launch is tile t % per_batch of problem
    // t / per_batch.  (mb, nb) are the problem's own blocks; problem p's A
    // and B are row blocks p * num_m + mb and p * num_n + nb of the stacked
    // operands (and of their scale planes).
    auto tile_coords = [&](int t, int& p, int& mb, int& nb) {
        p = t / per_batch;
        t -= p * per_batch;
        const int per_group = kGroup * num_n;
        const int g = t / per_group;
        const int first = g * kGroup;
        const int gsize = min(num_m - first, kGroup);
        const int r = t % per_group;
        mb = first + r % gsize;
        nb = r / gsize;
        // a routed launch starts its walk at another row block (see GemmArgs)
        if (args.rotate_m) {
            mb += args.rotate_m;
            if (mb >= num_m) mb -= num_m;
        }
    };

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- producer ----------------
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued[kStages] = {0};
            bool alive = true;
            for (int t = blockIdx.x; t < num_tiles && alive; t += gridDim.x) {
                int p, mb, nb;
                tile_coords(t, p, mb, nb);
                const int ga = p * num_m + mb, gb = p * num_n + nb;  // stacked row blocks
                // Scale atoms that exist: the last E2M1 stage of an odd atom
                // count has one, and B groups past the plane (a ragged N whose
                // last tile covers one 128-row group) have none.  The payload
                // boxes always count in full (TMA zero-fills past K).
                int b_groups_here = 0;
#pragma unroll
                for (int g = 0; g < BN / 128; ++g) b_groups_here += (gb * (BN / 128) + g < args.b_groups) ? 1 : 0;
                for (int ks = 0; ks < args.k_stages; ++ks) {
                    if (!ptx::mbar_wait(bar_empty + 8 * stage, phase ^ 1)) { alive = false; break; }
                    const uint32_t full = bar_full + 8 * stage;
                    const int64_t atom0 = int64_t(ks) * C::kAtoms;
                    const int atoms = ks + 1 < args.k_stages ? C::kAtoms : args.last_atoms;
                    ptx::mbar_arrive_expect_tx(full, C::kABytes + C::kBBytes + (1 + b_groups_here) * atoms * 512);
                    ptx::tma_load_2d(sbase + C::kOffA + stage * C::kABytes, &tmap_a, ks * kBKBytes, ga * kBM, full);
                    ptx::tma_load_2d(sbase + C::kOffB + stage * C::kBBytes, &tmap_b, ks * kBKBytes, gb * BN, full);
                    ptx::bulk_load(sbase + C::kOffSfa + stage * C::kSfaBytes,
                                   args.sfa + (int64_t(ga) * args.katoms + atom0) * 512, atoms * 512, full);
#pragma unroll
                    for (int g = 0; g < BN / 128; ++g) {
                        if (gb * (BN / 128) + g >= args.b_groups) continue;
                        ptx::bulk_load(sbase + C::kOffSfb + stage * C::kSfbBytes + g * C::kAtoms * 512,
                                       args.sfb + ((int64_t(gb) * (BN / 128) + g) * args.katoms + atom0) * 512,
                                       atoms * 512, full);
                    }
                    issued[stage] += 1;
                    if (++stage == kStages) { stage = 0; phase ^= 1; }
                }
            }
            // Let every copy this thread started land before the CTA can exit.
            for (int s = 0; s < kStages; ++s)
                if (issued[s] > 0) ptx::mbar_wait(bar_full + 8 * s, (issued[s] - 1) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            const uint32_t fmt_code = FMT == SW_MX_E4M3 ? 0u : 1u;
            int stage = 0;
            uint32_t phase = 0;
            uint32_t tile_iter = 0;
            bool alive = true;
            for (int t = blockIdx.x; t < num_tiles && alive; t += gridDim.x, ++tile_iter) {
                // the epilogue must have drained the accumulator of the previous tile
                if (!ptx::mbar_wait(bar_tmem_empty, (tile_iter & 1) ^ 1)) break;
                ptx::tc_fence_after();
                for (int ks = 0; ks < args.k_stages; ++ks) {
                    if (!ptx::mbar_wait(bar_full + 8 * stage, phase)) { alive = false; break; }
                    ptx::tc_fence_after();
                    const uint32_t sf_col = tmem + C::kSfCol0 + stage * C::kSfColsPerStage;
                    const uint32_t sfa_col = sf_col;
                    const uint32_t sfb_col = sf_col + C::kSfaCols;
                    const uint32_t a_addr = sbase + C::kOffA + stage * C::kABytes;
                    const uint32_t b_addr = sbase + C::kOffB + stage * C::kBBytes;
                    // One stage: its scale atoms into TMEM (shared memory -> TMEM,
                    // replicated per sub-partition), then its MMAs, 32 payload
                    // bytes of K each.  Full stages run with the counts as
                    // constants; only a ragged last stage passes fewer atoms
                    // (those the producer loaded) and MMAs (those reaching real K
                    // blocks).  A B group past the plane was not loaded: its
                    // stale scales only reach result columns past N, which are
                    // not stored.
                    auto issue = [&](auto atoms, auto mmas) {
#pragma unroll
                        for (int a = 0; a < C::kAtoms; ++a) {
                            if (a >= int(atoms)) break;
                            ptx::tc_cp_32x128b_x4(sfa_col + 4 * a,
                                                  ptx::smem_desc(sbase + C::kOffSfa + stage * C::kSfaBytes + a * 512,
                                                                 0, 128, ptx::kLayoutNone));
#pragma unroll
                            for (int g = 0; g < BN / 128; ++g)
                                ptx::tc_cp_32x128b_x4(
                                    sfb_col + a * 4 * (BN / 128) + 4 * g,
                                    ptx::smem_desc(sbase + C::kOffSfb + stage * C::kSfbBytes + (g * C::kAtoms + a) * 512,
                                                   0, 128, ptx::kLayoutNone));
                        }
#pragma unroll
                        for (int j = 0; j < C::kMmaPerStage; ++j) {
                            if (j >= int(mmas)) break;
                            const uint64_t adesc = ptx::smem_desc(a_addr + 32 * j, 0, 1024, ptx::kLayoutSwizzle128);
                            const uint64_t bdesc = ptx::smem_desc(b_addr + 32 * j, 0, 1024, ptx::kLayoutSwizzle128);
                            const uint32_t accumulate = (ks > 0 || j > 0) ? 1u : 0u;
                            if (FMT == SW_MX_E4M3) {
                                const uint32_t idesc = make_idesc(fmt_code, kBM, BN, uint32_t(j), uint32_t(j));
                                ptx::mma_mxf8f6f4(tmem + C::kAccCol, adesc, bdesc, idesc, accumulate, sfa_col,
                                                  sfb_col);
                            } else {
                                const int atom = j / 2;
                                const uint32_t sf_id = uint32_t((2 * j) % 4);
                                const uint32_t idesc = make_idesc(fmt_code, kBM, BN, sf_id, sf_id);
                                ptx::mma_mxf4(tmem + C::kAccCol, adesc, bdesc, idesc, accumulate, sfa_col + 4 * atom,
                                              sfb_col + atom * 4 * (BN / 128));
                            }
                        }
                    };
                    if (ks + 1 < args.k_stages || !args.ragged_k)
                        issue(Count<C::kAtoms>{}, Count<C::kMmaPerStage>{});
                    else
                        issue(args.last_atoms, args.last_mmas);
                    ptx::tc_commit(bar_empty + 8 * stage);  // frees the smem stage and its scale columns
                    if (++stage == kStages) { stage = 0; phase ^= 1; }
                }
                if (!alive) break;
                ptx::tc_commit(bar_tmem_full);
            }
            // Drain every MMA this thread issued before TMEM is released.
            ptx::tc_commit(bar_drain);
            ptx::mbar_wait(bar_drain, 0);
        }
    } else if (kEpi == kEpiBf16Rows) {
        // ---------------- epilogue, staged through shared memory ----------------
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;        // columns [128 half, 128 half + 128) of the tile
        const int row = quarter * 32 + lane;     // row of the tile this thread drains
        const bool leader = threadIdx.x == 64 + 128 * half;  // issues this half's stores
        uint8_t* stage_out = smem + C::kOffOut;
        const uint32_t stage_addr = sbase + C::kOffOut;
        // Every epilogue thread runs the same barrier sequence for every tile:
        // after a bounded wait gives up the thread stops working but keeps
        // meeting the named barriers, so no thread can wait for one that left.
        uint32_t tile_iter = 0;
        bool alive = true;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tile_iter) {
            int p, mb, nb;
            tile_coords(t, p, mb, nb);
            uint32_t w[4][16];  // the half's 128 columns as bf16 pairs
            if (alive && !ptx::mbar_wait(bar_tmem_full, tile_iter & 1)) alive = false;
            if (alive) {
                ptx::tc_fence_after();
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t r[32];
                    ptx::tmem_ld_32x32b_x32(tmem + C::kAccCol + (uint32_t(quarter * 32) << 16) + half * 128 + c * 32,
                                            r);
                    ptx::tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
                        w[c][e] = *reinterpret_cast<uint32_t*>(&h);
                    }
                }
                // the accumulator is in registers: the next tile may start
                ptx::tc_fence_before();
                ptx::mbar_arrive(bar_tmem_empty);
            }
            // the previous tile's stores of this half must have left its staging
            if (leader && alive) ptx::bulk_wait_group_read0();
            ptx::named_barrier(1 + half, 128);
            if (alive) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    // 32 columns = 64 bytes = four 16-byte units of a 128-byte
                    // row of column group chunk/2, swizzled by row % 8
                    const int chunk = half * 4 + c;
                    uint8_t* grp = stage_out + (chunk >> 1) * (kBM * 128) + row * 128;
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int unit = ((chunk & 1) * 4 + u) ^ (row & 7);
                        *reinterpret_cast<uint4*>(grp + unit * 16) =
                            make_uint4(w[c][4 * u], w[c][4 * u + 1], w[c][4 * u + 2], w[c][4 * u + 3]);
                    }
                }
                ptx::fence_proxy_async_smem();
            }
            ptx::named_barrier(1 + half, 128);
            if (leader && alive) {
#pragma unroll
                for (int g = 2 * half; g < 2 * half + 2; ++g)
                    if (nb * BN + g * 64 < args.N)  // boxes partly past M or N are clipped by TMA
                        ptx::tma_store_2d(&tmap_c, nb * BN + g * 64, (p * num_m + mb) * kBM,
                                          stage_addr + g * (kBM * 128));
                ptx::bulk_commit_group();
            }
        }
        if (leader) ptx::bulk_wait_group0();
    } else if (kEpi == kEpiF32Rows || kEpi == kEpiF32Cols) {
        // ---------------- epilogue, fp32 chunks staged through shared memory ----------------
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;        // chunks 4 half .. 4 half + 3 of the tile
        const int row = quarter * 32 + lane;     // row of the tile this thread drains
        const bool leader = threadIdx.x == 64 + 128 * half;  // issues this half's stores
        float* stage_out = reinterpret_cast<float*>(smem + C::kOffOut);
        const uint32_t stage_addr = sbase + C::kOffOut;
        // As in the bf16 epilogue, every thread meets the same named barriers for
        // every chunk even after a bounded wait has given up.  Each half rotates
        // through its own two of the kOutBufs chunk buffers.
        uint32_t tile_iter = 0;
        bool alive = true;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tile_iter) {
            int p, mb, nb;
            tile_coords(t, p, mb, nb);
            uint32_t r[4][32];
            if (alive && !ptx::mbar_wait(bar_tmem_full, tile_iter & 1)) alive = false;
            if (alive) {
                ptx::tc_fence_after();
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    ptx::tmem_ld_32x32b_x32(tmem + C::kAccCol + (uint32_t(quarter * 32) << 16) + half * 128 + c * 32,
                                            r[c]);
                ptx::tmem_ld_wait();
                // the accumulator is in registers: the next tile may start
                ptx::tc_fence_before();
                ptx::mbar_arrive(bar_tmem_empty);
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int chunk = half * 4 + c;
                const int buf = 2 * half + (c & 1);
                // the store that last read this buffer (two chunks ago) must be done with it
                if (leader && alive) ptx::bulk_wait_group_read<1>();
                ptx::named_barrier(1 + half, 128);
                if (alive) {
                    float* b = stage_out + buf * (kChunkBytes / 4);
                    if (kEpi == kEpiF32Cols) {
                        // [32 n][128 m]: the lanes of a warp write consecutive m
#pragma unroll
                        for (int e = 0; e < 32; ++e) b[e * kBM + row] = __uint_as_float(r[c][e]);
                    } else {
                        // [128 m][32 n], 16-byte units swizzled by m % 8 (the map's 128-byte swizzle)
                        float4* rowp = reinterpret_cast<float4*>(b + row * 32);
#pragma unroll
                        for (int u = 0; u < 8; ++u)
                            rowp[u ^ (row & 7)] =
                                make_float4(__uint_as_float(r[c][4 * u]), __uint_as_float(r[c][4 * u + 1]),
                                            __uint_as_float(r[c][4 * u + 2]), __uint_as_float(r[c][4 * u + 3]));
                    }
                    ptx::fence_proxy_async_smem();
                }
                ptx::named_barrier(1 + half, 128);
                if (kEpi == kEpiF32Rows && args.routed && alive) {
                    // Routed results: the half's 128 threads copy the staged
                    // chunk to its owner's block, a warp writing four whole
                    // 128-byte row segments per pass (full lines over NVLink),
                    // as streaming stores: evict-first in L2, so the 4 bytes
                    // per result do not push operand tiles out.
                    // The next write of this buffer waits at the named barrier
                    // above, which every thread meets after its reads here.
                    // Thread t moves 16-byte unit u = t % 8 of rows t / 8 + 16 i
                    // (i < 8): u and the swizzle (row % 8 = (t / 8) % 8) stay
                    // fixed, so each pass is one shared load and one store at
                    // constant strides.  N % 4 == 0: a unit is all in or out.
                    const int tid = threadIdx.x - (64 + 128 * half);
                    const int u = tid & 7, r0 = tid >> 3;
                    const int64_t n = int64_t(nb) * BN + chunk * 32 + 4 * u;
                    if (n < args.N) {
                        const int owner = int(int64_t(mb) * kBM / args.rows_per_dest);
                        const int64_t m0 = int64_t(mb) * kBM - int64_t(owner) * args.rows_per_dest + r0;
                        float* g = args.dest[owner] + m0 * args.ldc_m + n;
                        const int64_t g_step = 16 * args.ldc_m;
                        const float4* s = reinterpret_cast<const float4*>(stage_out + buf * (kChunkBytes / 4) +
                                                                          r0 * 32) + (u ^ (r0 & 7));
                        const int rows_left = args.M - mb * kBM - r0;  // whole tiles in a routed launch
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            if (16 * i < rows_left) __stcs(reinterpret_cast<float4*>(g + i * g_step), s[i * 128]);
                    }
                } else if (leader && alive) {
                    // A chunk wholly past N (a ragged last tile) stores nothing,
                    // but still commits a (then empty) group: the buffer-reuse
                    // wait above counts one group per chunk.  Partial boxes are
                    // clipped by TMA.
                    if (nb * BN + chunk * 32 < args.N) {
                        const uint32_t src = stage_addr + buf * kChunkBytes;
                        if (kEpi == kEpiF32Cols)
                            ptx::tma_store_2d(&tmap_c, mb * kBM, (p * num_n + nb) * BN + chunk * 32, src);
                        else
                            ptx::tma_store_2d(&tmap_c, nb * BN + chunk * 32, (p * num_m + mb) * kBM, src);
                    }
                    ptx::bulk_commit_group();
                }
            }
        }
        if (leader) ptx::bulk_wait_group0();
        // routed results went to other GPUs: performed at system scope before
        // the thread finishes (the signal that follows the kernel publishes them)
        if (kEpi == kEpiF32Rows && args.routed) __threadfence_system();
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int quarter = warp & 3;  // TMEM sub-partition this warp may access
        const int row_in_tile = quarter * 32 + lane;
        uint32_t tile_iter = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tile_iter) {
            int p, mb, nb;
            tile_coords(t, p, mb, nb);
            if (!ptx::mbar_wait(bar_tmem_full, tile_iter & 1)) break;
            ptx::tc_fence_after();
            const int64_t m_tile = int64_t(mb) * kBM + row_in_tile;
            const bool row_in = m_tile < args.M;  // the last tile row of a ragged M reaches past it
#pragma unroll 1
            for (int chunk = 0; chunk < BN / 32; ++chunk) {
                uint32_t r[32];
                ptx::tmem_ld_32x32b_x32(tmem + C::kAccCol + (uint32_t(quarter * 32) << 16) + chunk * 32, r);
                ptx::tmem_ld_wait();
                const int64_t n0 = int64_t(nb) * BN + chunk * 32;
                if (!row_in || n0 >= args.N) continue;
                const int ncols = (int)min(int64_t(32), int64_t(args.N) - n0);  // < 32 only in the last column chunk
                if (args.out_bf16) {
                    const int64_t m = m_tile;
                    __nv_bfloat16* cptr = static_cast<__nv_bfloat16*>(args.c) + p * args.c_batch;
                    if (ncols == 32 && args.ldc_n == 1 && (((m * args.ldc_m + n0) & 7) == 0) &&
                        ((reinterpret_cast<uintptr_t>(cptr) & 15) == 0)) {
                        uint4* dst = reinterpret_cast<uint4*>(cptr + m * args.ldc_m + n0);
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            float f[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                f[e] = __uint_as_float(r[8 * v + e]);
                                if (args.beta_one) f[e] += __bfloat162float(cptr[m * args.ldc_m + n0 + 8 * v + e]);
                            }
                            __nv_bfloat162 h[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
                            dst[v] = *reinterpret_cast<uint4*>(h);
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            if (e >= ncols) break;
                            __nv_bfloat16* p = cptr + m * args.ldc_m + (n0 + e) * args.ldc_n;
                            float f = __uint_as_float(r[e]);
                            if (args.beta_one) f += __bfloat162float(*p);
                            *p = __float2bfloat16_rn(f);
                        }
                    }
                } else {
                    float* cptr = static_cast<float*>(args.c) + p * args.c_batch;
                    int64_t m = m_tile;
                    if (args.routed) {
                        // the tile's rows belong to one owner: its block starts at dest[owner]
                        const int owner = int(int64_t(mb) * kBM / args.rows_per_dest);
                        cptr = args.dest[owner];
                        m -= int64_t(owner) * args.rows_per_dest;
                    }
                    if (ncols == 32 && args.ldc_n == 1 && (((m * args.ldc_m + n0) & 3) == 0) &&
                        ((reinterpret_cast<uintptr_t>(cptr) & 15) == 0)) {
                        float4* dst = reinterpret_cast<float4*>(cptr + m * args.ldc_m + n0);
#pragma unroll
                        for (int v = 0; v < 8; ++v) {
                            float4 o = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                                   __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
                            if (args.beta_one) {
                                const float4 old = dst[v];
                                o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
                            }
                            dst[v] = o;
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            if (e >= ncols) break;
                            float* p = cptr + m * args.ldc_m + (n0 + e) * args.ldc_n;
                            float f = __uint_as_float(r[e]);
                            if (args.beta_one) f += *p;
                            *p = f;
                        }
                    }
                }
            }
            ptx::tc_fence_before();
            ptx::mbar_arrive(bar_tmem_empty);
        }
        // routed results went to other GPUs too: have them performed at
        // system scope before this thread finishes (the signal that follows
        // the kernel on its stream publishes them)
        if (args.routed) __threadfence_system();
    }

    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    if (warp == 1) ptx::tmem_dealloc(tmem, kTmemCols);
}

// ---- host side -------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() { return tensor_map_encoder(); }

// 2-D bf16 map over C (rows x cols, row pitch ld_bytes), box 64 x 128 with the
// 128-byte swizzle of the epilogue's staging tile.
int make_output_map(CUtensorMap* map, void* base, int64_t rows, int64_t cols, int64_t ld_bytes) {
    auto fn = encode_fn();
    if (!fn) return fail(SW_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld_bytes};
    cuuint32_t box[2] = {64, (cuuint32_t)kBM};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SW_ERR_INVALID, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
    return SW_OK;
}

// 2-D fp32 map over an outer x inner matrix (row pitch ld_bytes), box
// box_inner x box_outer, 128-byte swizzle when `swizzle` (a 32-float inner box).
int make_output_map_f32(CUtensorMap* map, void* base, int64_t outer, int64_t inner, int64_t ld_bytes,
                        uint32_t box_inner, uint32_t box_outer, bool swizzle) {
    auto fn = encode_fn();
    if (!fn) return fail(SW_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)ld_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SW_ERR_INVALID, "cuTensorMapEncodeTiled (fp32 output) failed (%d)", (int)r);
    return SW_OK;
}

// 2-D uint8 map over rows x row_bytes (pitch ld), box 128 bytes x box_rows,
// 128-byte swizzle (the canonical K-major layout of the UMMA descriptors).
int make_operand_map(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes, int64_t ld,
                     uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return fail(SW_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld};
    cuuint32_t box[2] = {(cuuint32_t)kBKBytes, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SW_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return SW_OK;
}

template <int FMT, int BN, int kStages, int kEpi>
int launch_gemm(const uint8_t* a, int64_t lda, const uint8_t* sfa, const uint8_t* b, int64_t ldb,
                const uint8_t* sfb, void* c, int out_dtype, int64_t ldc_m, int64_t ldc_n, int64_t M, int64_t N,
                int64_t K, int beta_one, int64_t batch, int64_t c_batch, int max_ctas, cudaStream_t stream,
                const Route* route) {
    using Cf = Cfg<FMT, BN, kStages, kEpi>;
    const int64_t row_bytes = FMT == SW_MX_E4M3 ? K : K / 2;
    // the maps cover the stacked operands (batch * M rows of A, batch * N of B)
    // and, for the staged epilogues, the stacked results
    CUtensorMap ma, mb;
    int rc = make_operand_map(&ma, a, batch * M, row_bytes, lda, kBM);
    if (rc != SW_OK) return rc;
    rc = make_operand_map(&mb, b, batch * N, row_bytes, ldb, BN);
    if (rc != SW_OK) return rc;
    CUtensorMap mc;
    memset(&mc, 0, sizeof(mc));
    if (kEpi == kEpiBf16Rows) rc = make_output_map(&mc, c, batch * M, N, ldc_m * 2);
    if (kEpi == kEpiF32Rows) rc = make_output_map_f32(&mc, c, batch * M, N, ldc_m * 4, 32, kBM, true);
    if (kEpi == kEpiF32Cols) rc = make_output_map_f32(&mc, c, batch * N, M, ldc_n * 4, kBM, 32, false);
    if (rc != SW_OK) return rc;
    GemmArgs args;
    args.sfa = sfa;
    args.sfb = sfb;
    args.c = c;
    args.ldc_m = ldc_m;
    args.ldc_n = ldc_n;
    args.M = (int)M;
    args.N = (int)N;
    args.K = (int)K;
    args.k_stages = (int)((row_bytes + kBKBytes - 1) / kBKBytes);
    args.katoms = (int)((K / 32 + 3) / 4);
    args.row_bytes = (int)row_bytes;
    args.b_groups = (int)((batch * N + 127) / 128);
    args.last_atoms = args.katoms - (args.k_stages - 1) * Cf::kAtoms;
    args.last_mmas = (int)((row_bytes - int64_t(args.k_stages - 1) * kBKBytes + 31) / 32);
    args.ragged_k = args.last_atoms != Cf::kAtoms || args.last_mmas != Cf::kMmaPerStage;
    args.beta_one = beta_one;
    args.out_bf16 = out_dtype == SW_OUT_BF16;
    args.batch = (int)batch;
    args.c_batch = c_batch;
    args.routed = route != nullptr;
    args.rows_per_dest = route ? route->rows_per_dest : 0;
    for (int q = 0; q < kMaxRouted; ++q) args.dest[q] = route && q < route->count ? route->dest[q] : nullptr;
    args.rotate_m = route ? (int)((int64_t(route->first) * route->rows_per_dest / kBM) % ((M + kBM - 1) / kBM)) : 0;
    auto kernel = mx_gemm_kernel<FMT, BN, kStages, kEpi>;
    SW_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::kSmemBytes),
                "set gemm smem");
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t tiles = batch * ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
    int grid = (int)std::min<int64_t>(tiles, sms);
    if (max_ctas > 0) grid = std::min(grid, max_ctas);  // leave SMs to concurrent work (a collective)
    SW_CUDA_TRY(launch_pdl(kernel, grid, Cf::kThreads, Cf::kSmemBytes, stream, ma, mb, mc, args), "mx_gemm launch");
    SW_LAUNCH_CHECK("mx_gemm launch");
    return SW_OK;
}

}  // namespace
}  // namespace sw

namespace sw {
namespace {

// Checks and dispatch shared by the entry points; `batch` problems stacked as
// described at sw_mx_gemm_batched (1 for one contraction).
int mx_gemm_impl(int fmt_a, int fmt_b, const uint8_t* a, int64_t lda, const uint8_t* scales_a, const uint8_t* b,
                 int64_t ldb, const uint8_t* scales_b, void* c, int out_dtype, int64_t ldc_m, int64_t ldc_n,
                 int64_t M, int64_t N, int64_t K, int beta_one, int64_t batch, int64_t c_batch, int max_ctas,
                 void* stream, const Route* route = nullptr) {
    if (fmt_a != fmt_b) return fail(SW_ERR_UNSUPPORTED, "sw_mx_gemm: mixed operand formats are not supported");
    if (fmt_a != SW_MX_E4M3 && fmt_a != SW_MX_E2M1) return fail(SW_ERR_INVALID, "sw_mx_gemm: unknown format %d", fmt_a);
    if (out_dtype != SW_OUT_F32 && out_dtype != SW_OUT_BF16)
        return fail(SW_ERR_INVALID, "sw_mx_gemm: unknown output dtype %d", out_dtype);
    if (M < 0 || N < 0 || K < 0) return fail(SW_ERR_INVALID, "sw_mx_gemm: negative extent");
    if (M == 0 || N == 0) return ok();
    if (!a || !b || !scales_a || !scales_b || !c) return fail(SW_ERR_INVALID, "sw_mx_gemm: null pointer");
    // Any M and N: the last tile row / column reaches past them, its operand
    // rows are zero-filled by TMA and its results past M / N are not stored.
    // K runs in whole 32-element MX blocks; past K the payload boxes are
    // zero-filled and only the MMAs that reach real blocks are issued.
    if (K % 32 != 0 || K == 0)
        return fail(SW_ERR_UNSUPPORTED, "sw_mx_gemm: needs K to be a positive multiple of 32 (got %lld x %lld x %lld)",
                    (long long)M, (long long)N, (long long)K);
    if (batch > 1 && (M % 128 != 0 || N % 128 != 0))
        return fail(SW_ERR_UNSUPPORTED,
                    "sw_mx_gemm_batched: needs M %% 128 == 0 and N %% 128 == 0 (got %lld x %lld)", (long long)M,
                    (long long)N);
    if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return fail(SW_ERR_UNSUPPORTED, "sw_mx_gemm: extent too large");
    if (batch < 1 || c_batch < 0) return fail(SW_ERR_INVALID, "sw_mx_gemm: bad batch count or result stride");
    if (batch * M > INT32_MAX || batch * N > INT32_MAX || batch * ((M + 127) / 128) * ((N + 127) / 128) > INT32_MAX)
        return fail(SW_ERR_UNSUPPORTED, "sw_mx_gemm: stacked extent too large");
    const int64_t row_bytes = fmt_a == SW_MX_E4M3 ? K : K / 2;
    if (lda < row_bytes || ldb < row_bytes || lda % 16 != 0 || ldb % 16 != 0)
        return fail(SW_ERR_INVALID, "sw_mx_gemm: payload pitches must cover a row and be multiples of 16 bytes");
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(scales_a) |
         reinterpret_cast<uintptr_t>(scales_b)) & 15)
        return fail(SW_ERR_INVALID, "sw_mx_gemm: payload and scale planes must be 16-byte aligned");
    if (ldc_m < 1 || ldc_n < 1) return fail(SW_ERR_INVALID, "sw_mx_gemm: output pitches must be positive");
    // Stacked results must not overlap: CTAs of different problems store (and,
    // with beta_one, read back) their tiles concurrently.  The (problem, m, n)
    // -> element map is injective when, taking its three modes in order of
    // stride, each stride exceeds the span of the modes below it; this admits
    // stacked blocks and interleaved problems (a batch mode of stride 1) alike.
    if (batch > 1) {
        int64_t ext[3] = {batch, M, N}, str[3] = {c_batch, ldc_m, ldc_n};
        for (int i = 0; i < 3; ++i)
            for (int j = i + 1; j < 3; ++j)
                if (str[j] < str[i]) { std::swap(str[i], str[j]); std::swap(ext[i], ext[j]); }
        int64_t span = 0;
        bool disjoint = true;
        for (int i = 0; i < 3; ++i) {
            if (ext[i] == 1) continue;
            if (str[i] <= span) disjoint = false;
            span += (ext[i] - 1) * str[i];
        }
        if (!disjoint)
            return fail(SW_ERR_INVALID,
                        "sw_mx_gemm_batched: results of the stacked problems may overlap (batch_stride_c %lld, "
                        "ldc_m %lld, ldc_n %lld)",
                        (long long)c_batch, (long long)ldc_m, (long long)ldc_n);
    }
    if (max_ctas < 0) return fail(SW_ERR_INVALID, "sw_mx_gemm: max_ctas must be >= 0 (0 = every SM)");
    cudaStream_t s = (cudaStream_t)stream;
    // Results without accumulation, with a unit pitch on either side, take a
    // staged TMA epilogue (3 mainloop stages + the staging buffers); anything
    // else stores straight from registers (4 stages).
    const bool aligned_c = (reinterpret_cast<uintptr_t>(c) & 15) == 0;
    const int esize = out_dtype == SW_OUT_BF16 ? 2 : 4;
    int epi = kEpiDirect;
    // 128 x 256 tiles unless the last one would be at most half used (then
    // 128 x 128 tiles), and for stacked problems only whole 256-column tiles;
    // a ragged last tile is clipped
    const bool wide = N % 256 == 0 || (batch == 1 && N % 256 > 128);
    // (a batched launch stages its results only when they stack without gaps)
    if (route && wide) {
        // routed: the staged chunks leave shared memory as whole row segments
        epi = kEpiF32Rows;
    } else if (!beta_one && wide && aligned_c && !route) {
        if (ldc_n == 1 && (ldc_m * esize) % 16 == 0 && ldc_m >= N && (batch == 1 || c_batch == M * ldc_m))
            epi = out_dtype == SW_OUT_BF16 ? kEpiBf16Rows : kEpiF32Rows;
        else if (out_dtype == SW_OUT_F32 && ldc_m == 1 && (ldc_n * 4) % 16 == 0 && ldc_n >= M &&
                 (batch == 1 || c_batch == N * ldc_n))
            epi = kEpiF32Cols;
    }
    int rc;
#define SW_GEMM(F, BNV, ST, EPI) \
    launch_gemm<F, BNV, ST, EPI>(a, lda, scales_a, b, ldb, scales_b, c, out_dtype, ldc_m, ldc_n, M, N, K, beta_one, \
                                 batch, c_batch, max_ctas, s, route)
#define SW_GEMM_FMT(F)                                                                  \
    (epi == kEpiBf16Rows  ? SW_GEMM(F, 256, 3, kEpiBf16Rows)                             \
     : epi == kEpiF32Rows ? SW_GEMM(F, 256, 3, kEpiF32Rows)                              \
     : epi == kEpiF32Cols ? SW_GEMM(F, 256, 3, kEpiF32Cols)                              \
     : wide               ? SW_GEMM(F, 256, 4, kEpiDirect)                               \
                          : SW_GEMM(F, 128, 4, kEpiDirect))
    rc = fmt_a == SW_MX_E4M3 ? SW_GEMM_FMT(SW_MX_E4M3) : SW_GEMM_FMT(SW_MX_E2M1);
#undef SW_GEMM_FMT
#undef SW_GEMM
    if (rc != SW_OK) return rc;
    return ok();
}

}  // namespace
}  // namespace sw

extern "C" int sw_mx_gemm_ex(int fmt_a, int fmt_b, const uint8_t* a, int64_t lda, const uint8_t* scales_a,
                             const uint8_t* b, int64_t ldb, const uint8_t* scales_b, void* c, int out_dtype,
                             int64_t ldc_m, int64_t ldc_n, int64_t M, int64_t N, int64_t K, int beta_one,
                             int max_ctas, void* stream) {
    return sw::mx_gemm_impl(fmt_a, fmt_b, a, lda, scales_a, b, ldb, scales_b, c, out_dtype, ldc_m, ldc_n, M, N, K,
                            beta_one, 1, 0, max_ctas, stream);
}

extern "C" int sw_mx_gemm_batched(int fmt_a, int fmt_b, const uint8_t* a, int64_t lda, const uint8_t* scales_a,
                                  const uint8_t* b, int64_t ldb, const uint8_t* scales_b, void* c, int out_dtype,
                                  int64_t ldc_m, int64_t ldc_n, int64_t batch_stride_c, int64_t batch, int64_t M,
                                  int64_t N, int64_t K, int beta_one, void* stream) {
    if (batch == 0) return sw::ok();
    return sw::mx_gemm_impl(fmt_a, fmt_b, a, lda, scales_a, b, ldb, scales_b, c, out_dtype, ldc_m, ldc_n, M, N, K,
                            beta_one, batch, batch_stride_c, 0, stream);
}

extern "C" int sw_mx_gemm_routed(int fmt, const uint8_t* a, int64_t lda, const uint8_t* scales_a, const uint8_t* b,
                                 int64_t ldb, const uint8_t* scales_b, float* const* dest, int ndest,
                                 int64_t rows_per_dest, int64_t ldc, int first, int64_t M, int64_t N, int64_t K,
                                 int max_ctas, void* stream) {
    using namespace sw;
    if (ndest < 1 || ndest > kMaxRouted)
        return fail(SW_ERR_INVALID, "sw_mx_gemm_routed: 1 to %d destinations (got %d)", kMaxRouted, ndest);
    if (!dest) return fail(SW_ERR_INVALID, "sw_mx_gemm_routed: null destination list");
    if (rows_per_dest <= 0 || rows_per_dest % 128 != 0 || rows_per_dest * ndest != M)
        return fail(SW_ERR_INVALID,
                    "sw_mx_gemm_routed: the %d destinations must each take whole 128-row tiles, M = %lld rows in all",
                    ndest, (long long)M);
    if (ldc < N || ldc % 4 != 0 || N % 4 != 0)
        return fail(SW_ERR_INVALID, "sw_mx_gemm_routed: N must be a multiple of 4 and ldc cover N, a multiple of 4");
    if (first < 0 || first >= ndest)
        return fail(SW_ERR_INVALID, "sw_mx_gemm_routed: the first destination must be one of the %d (got %d)", ndest,
                    first);
    Route route;
    route.count = ndest;
    route.rows_per_dest = rows_per_dest;
    route.first = first;
    for (int q = 0; q < ndest; ++q) {
        if (!dest[q] || (reinterpret_cast<uintptr_t>(dest[q]) & 15))
            return fail(SW_ERR_INVALID, "sw_mx_gemm_routed: destination %d is null or not 16-byte aligned", q);
        route.dest[q] = dest[q];
    }
    return mx_gemm_impl(fmt, fmt, a, lda, scales_a, b, ldb, scales_b, dest[0], SW_OUT_F32, ldc, 1, M, N, K, 0, 1, 0,
                        max_ctas, stream, &route);
}

extern "C" int sw_mx_gemm(int fmt_a, int fmt_b, const uint8_t* a, int64_t lda, const uint8_t* scales_a,
                          const uint8_t* b, int64_t ldb, const uint8_t* scales_b, void* c, int out_dtype,
                          int64_t ldc_m, int64_t ldc_n, int64_t M, int64_t N, int64_t K, int beta_one,
                          void* stream) {
    return sw_mx_gemm_ex(fmt_a, fmt_b, a, lda, scales_a, b, ldb, scales_b, c, out_dtype, ldc_m, ldc_n, M, N, K,
                         beta_one, 0, stream);
}
