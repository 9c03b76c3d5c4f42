// Q4_0 x Q8_0 for rows > 4 (the reference's MX path) on the 5th-generation tensor cores.
//
// The reference's tiled Q4_0 x Q8_0 program (src/qpu_xla/kernels/ggml_q4_0.py:310-547, prepared by
// qpu_llama_q4_0.c:238-290 for rows > 4, EXACT weight mode) keeps one fp32 accumulator per output
// and adds the blocks in order: acc += ((float)dot_b * d_a[m, b]) * d_w[n, b] (itof, fmul by the
// activation scale, fmul by the weight scale, fadd; ggml_q4_0.py:506-513). Every block's integer
// dot has to reach the fp32 arithmetic on its own, so the K reduction cannot stay inside the
// tensor core: each 32-deep block is one tcgen05.mma (s8 x s8 -> s32, K = 32) into its own
// tensor-memory slot, and the epilogue warps drain the slots block by block.
//
// Orientation: the MMA's M side is 128 weight columns (tensor-memory lanes) and its N side is R
// activation rows (tensor-memory columns), R = 16, 32, 64 or 128 by the call's row count, so a
// call with few rows computes no padded rows: at 16 rows a tile is 128 x 16 outputs.
//
// Operands (prepared once): the weight codes expanded to int8 (code - 8), K-major rows of
// blocks_pad * 32 bytes, and the fp32 weight scales block-major [blocks_pad][columns]; per call the
// split activation (int8 rows of blocks_pad * 32 bytes, zero-padded) and its fp32 scales
// block-major [blocks_pad][rows_pad]. TMA moves a stage of four blocks of each (the two int8 tiles
// in the 128-byte swizzle the MMA descriptors read, the two scale boxes plain).
//
// Exact (float)dot without a conversion instruction (an int-to-float convert runs at a quarter of
// the fp32 rate): the MMA overwrites its slot with the s32 dot, and the epilogue adds the int32
// bits of 1.5 * 2^23 (0x4B400000) to it with one integer add, which gives the float bits of
// 1.5 * 2^23 + dot (|dot| <= 32 * 8 * 128 < 2^22, one ulp = 1); one fp32 subtraction of
// 1.5 * 2^23 then gives (float)dot exactly.
//
// Warps: 0 TMA producer, 1 tensor-memory allocator and MMA issuer (one thread), then 4 * G epilogue
// warps. Epilogue warp w reads the lanes of its quarter (w % 4: 32 weight columns, one per thread)
// and the rows of its group ((w - 2) / 4: R / G rows), keeping R / G fp32 accumulators per thread;
// the thread's weight scale is one word per block and the rows' activation scales are broadcast
// reads. Stage reuse waits for the MMA commit and for every epilogue thread (they read the stage's
// scales); a slot is free again once every epilogue thread has loaded its words, before their fp32
// work on them. Every mbarrier wait is bounded.
#include <cuda_fp16.h>

#include <cstring>

#include "qpucuda_internal.h"
#include "sm100_sync.cuh"


namespace qpucuda {
namespace {

constexpr int kBW = 128;   // weight columns per tile (MMA M, tensor-memory lanes)
constexpr int kKB = 4;     // Q4_0 blocks per stage: 128 bytes of K
constexpr int kSlots = 4;  // tensor-memory slots, one per block of a stage
constexpr uint32_t kMagicBits = 0x4B400000u;  // 1.5 * 2^23
constexpr float kMagic = 12582912.0f;

constexpr int round_up(int value, int step) { return (value + step - 1) / step * step; }
constexpr uint32_t tmem_columns(uint32_t need) {
    uint32_t cols = 32;
    while (cols < need) cols *= 2;
    return cols;
}

// R activation rows per tile (MMA N), G epilogue warp groups.
template <int R, int G>
struct MxShape {
    static_assert(R % 16 == 0 && R >= 16 && R <= 128, "MMA N for M = 128");
    static constexpr int kEpilogueWarps = 4 * G;
    static constexpr int kThreads = 64 + 32 * kEpilogueWarps;
    static constexpr int kCols = R / G;  // rows (tensor-memory columns) per epilogue thread
    static_assert(kCols % 4 == 0, "scale reads go four rows at a time");
    static constexpr int kWidth = kCols < 16 ? kCols : 16;  // words per tensor-memory load
    static constexpr int kChunks = kCols / kWidth;
    static constexpr int kTileW = kBW * 128;
    static constexpr int kTileA = R * 128;
    static constexpr int kTileDw = kKB * kBW * 4;
    static constexpr int kTileDa = kKB * R * 4;
    static constexpr int kTxBytes = kTileW + kTileA + kTileDw + kTileDa;
    static constexpr int kStageBytes = round_up(kTxBytes, 1024);
    // Narrow tiles run two CTAs per SM (their epilogues interleave; a 70B projection at 16 rows
    // then fits in one wave); the shared-memory ring is sized for that.
    static constexpr int kCtasPerSm = R <= 32 ? 2 : 1;
    static constexpr int kRingBudget = 200 * 1024 / kCtasPerSm;
    static constexpr int kStages = kRingBudget / kStageBytes < 8 ? kRingBudget / kStageBytes : 8;
    static constexpr uint32_t kTmemCols = tmem_columns(kSlots * R);
    // D = s32, A = s8, B = s8, both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
    static constexpr uint32_t kInstrDesc =
        (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(R >> 3) << 17) | (static_cast<uint32_t>(kBW >> 4) << 24);
};

template <int kStages>
struct Control {
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t slot_full[kSlots];
    uint64_t slot_empty[kSlots];
    uint64_t drain;
    uint32_t tmem_base;
    volatile int abort_flag;
};

template <int R, int G>
constexpr size_t smem_bytes() {
    using S = MxShape<R, G>;
    return static_cast<size_t>(S::kStages) * S::kStageBytes + 1024 + sizeof(Control<S::kStages>);
}

struct MxParams {
    uint32_t rows;      // outputs are written for rows < rows
    uint32_t k_stages;  // blocks_pad / kKB
    uint32_t m_tiles, n_tiles;
    uint32_t col0;      // first weight column of the call (within the resident window)
    uint32_t count;     // columns computed
    uint32_t out_col0;  // destination column of weight column col0
    float *destination;
    size_t destination_stride;
    unsigned int *error_word;
};

using namespace sm100;

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t address) {
    // start >> 4 (bits 0-13), leading byte offset 16 B (unused for swizzled K-major), stride byte
    // offset 1024 B (8 rows of 128 B), descriptor version 1, 128-byte swizzle.
    return static_cast<uint64_t>((address & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) | (static_cast<uint64_t>(2) << 61);
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t instr_desc) {
    // overwrite the slot (enable-input-d = false): it holds this block's dot alone
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(instr_desc)
        : "memory");
}

__device__ __forceinline__ void commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 lanes x W columns of 32-bit words from tensor memory; the caller waits with tmem_wait_ld,
// which names the registers so nothing reads them before the load has landed.
template <int W>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[W]);
template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t taddr, uint32_t (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
template <int W>
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[W]) {
    // an empty asm that names the registers as read-write keeps every use after the wait
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < W; ++i) asm volatile("" : "+r"(r[i]));
}

__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
    return static_cast<unsigned long long>(__float_as_uint(lo)) | (static_cast<unsigned long long>(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// W rows of one block for the thread's weight column: acc[j] += (((float)dot_j) * da[j]) * dw, in
// that rounding order. r holds the slot words (s32 dots), da the rows' activation scales in shared
// memory (the same address in every lane: a broadcast), dw the column's weight scale. The
// subtraction and the two multiplies run on packed pairs (each half rounded exactly as __fadd_rn /
// __fmul_rn); the accumulation is a scalar __fadd_rn per output.
template <int W>
__device__ __forceinline__ void accumulate(float *acc, const uint32_t (&r)[W], const float *da, float dw) {
    const unsigned long long minus_magic = pack2(-kMagic, -kMagic);
    const unsigned long long dw2 = pack2(dw, dw);
#pragma unroll
    for (int q = 0; q < W / 4; ++q) {
        const float4 a = *reinterpret_cast<const float4 *>(da + 4 * q);
        unsigned long long lo = add2(pack2(__uint_as_float(r[4 * q] + kMagicBits), __uint_as_float(r[4 * q + 1] + kMagicBits)), minus_magic);
        unsigned long long hi = add2(pack2(__uint_as_float(r[4 * q + 2] + kMagicBits), __uint_as_float(r[4 * q + 3] + kMagicBits)), minus_magic);
        lo = mul2(mul2(lo, pack2(a.x, a.y)), dw2);
        hi = mul2(mul2(hi, pack2(a.z, a.w)), dw2);
        acc[4 * q] = __fadd_rn(acc[4 * q], __uint_as_float(static_cast<uint32_t>(lo)));
        acc[4 * q + 1] = __fadd_rn(acc[4 * q + 1], __uint_as_float(static_cast<uint32_t>(lo >> 32)));
        acc[4 * q + 2] = __fadd_rn(acc[4 * q + 2], __uint_as_float(static_cast<uint32_t>(hi)));
        acc[4 * q + 3] = __fadd_rn(acc[4 * q + 3], __uint_as_float(static_cast<uint32_t>(hi >> 32)));
    }
}

template <int R, int G>
__global__ void __launch_bounds__(MxShape<R, G>::kThreads, MxShape<R, G>::kCtasPerSm)
    q4_0_mx_sm100_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                         const __grid_constant__ CUtensorMap map_da, const __grid_constant__ CUtensorMap map_dw,
                         const MxParams p) {
    using S = MxShape<R, G>;
    constexpr int kStages = S::kStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    auto *control = reinterpret_cast<Control<kStages> *>(smem + kStages * S::kStageBytes);
    auto stage_w = [&](uint32_t s) { return smem + s * S::kStageBytes; };
    auto stage_a = [&](uint32_t s) { return smem + s * S::kStageBytes + S::kTileW; };
    auto stage_dw = [&](uint32_t s) {
        return reinterpret_cast<const float *>(smem + s * S::kStageBytes + S::kTileW + S::kTileA);
    };
    auto stage_da = [&](uint32_t s) {
        return reinterpret_cast<const float *>(smem + s * S::kStageBytes + S::kTileW + S::kTileA + S::kTileDw);
    };

    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t tiles = p.m_tiles * p.n_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&control->full[s]), 1);
            mbar_init(smem_u32(&control->empty[s]), 1 + 32 * S::kEpilogueWarps);  // the MMA commit + every epilogue thread
        }
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(smem_u32(&control->slot_full[s]), 1);
            mbar_init(smem_u32(&control->slot_empty[s]), 32 * S::kEpilogueWarps);
        }
        mbar_init(smem_u32(&control->drain), 1);
        control->abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&control->tmem_base)),
                     "r"(S::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem_base = control->tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            prefetch_tensor_map(&map_a);
            prefetch_tensor_map(&map_w);
            prefetch_tensor_map(&map_da);
            prefetch_tensor_map(&map_dw);
            uint32_t stage = 0, phase = 0, issued_mask = 0, issued_phases = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
                const int m0 = static_cast<int>((tile % p.m_tiles) * R);
                const int n0 = static_cast<int>(p.col0 + (tile / p.m_tiles) * kBW);
                for (uint32_t ks = 0; ks < p.k_stages; ++ks) {
                    if (!wait_bounded_suspend(smem_u32(&control->empty[stage]), phase ^ 1u, &control->abort_flag, p.error_word)) {
                        ok = false;
                        break;
                    }
                    const uint32_t full = smem_u32(&control->full[stage]);
                    mbar_expect_tx(full, S::kTxBytes);
                    tma_load_2d(smem_u32(stage_w(stage)), &map_w, full, static_cast<int>(ks * 128), n0);
                    tma_load_2d(smem_u32(stage_a(stage)), &map_a, full, static_cast<int>(ks * 128), m0);
                    tma_load_2d(smem_u32(stage_dw(stage)), &map_dw, full, n0, static_cast<int>(ks * kKB));
                    tma_load_2d(smem_u32(stage_da(stage)), &map_da, full, m0, static_cast<int>(ks * kKB));
                    issued_mask |= 1u << stage;
                    issued_phases = (issued_phases & ~(1u << stage)) | (phase << stage);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                for (int s = 0; s < kStages; ++s)
                    if ((issued_mask >> s) & 1u) wait_drain(smem_u32(&control->full[s]), (issued_phases >> s) & 1u);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer: one MMA per block, block b of a stage into slot b ----------------
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, slot_phase = 0;
            bool ok = true, any = false;
            for (uint32_t tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
                for (uint32_t ks = 0; ok && ks < p.k_stages; ++ks) {
                    ok = wait_bounded_suspend(smem_u32(&control->full[stage]), phase, &control->abort_flag, p.error_word);
                    if (!ok) break;
                    fence_after();
                    const uint64_t w_desc = smem_desc_sw128(smem_u32(stage_w(stage)));
                    const uint64_t a_desc = smem_desc_sw128(smem_u32(stage_a(stage)));
#pragma unroll 1
                    for (uint32_t b = 0; b < kKB; ++b) {
                        ok = wait_bounded_suspend(smem_u32(&control->slot_empty[b]), slot_phase ^ 1u, &control->abort_flag,
                                                  p.error_word);
                        if (!ok) break;
                        fence_after();
                        // block b starts 32 bytes further along the swizzled 128-byte rows
                        mma_i8(tmem_base + b * R, w_desc + 2u * b, a_desc + 2u * b, S::kInstrDesc);
                        commit(smem_u32(&control->slot_full[b]));
                        any = true;
                    }
                    if (!ok) break;
                    commit(smem_u32(&control->empty[stage]));  // this stage's MMAs are done reading it
                    slot_phase ^= 1u;
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok && any) {
                commit(smem_u32(&control->drain));
                wait_drain(smem_u32(&control->drain), 0);
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: drain, scale and accumulate, block by block ----------------
        // Software pipeline over loads of kWidth words, alternating between two register buffers:
        // while one load's fp32 work runs, the next load is in flight -- the block's next chunk, or
        // the following block's first one (once its slot is full). Block b of a stage always lands
        // in slot b (every tile has whole stages), so the four blocks of a stage unroll with fixed
        // slot addresses and scale offsets. Padding blocks need no test: their values and both
        // scales are zero, and adding the +0 or -0 they produce leaves every sum unchanged (a sum
        // that starts at +0 never becomes -0 under round-to-nearest).
        constexpr int kW = S::kWidth;
        const uint32_t quarter = warp & 3u;
        const uint32_t group = (warp - 2u) >> 2;
        const uint32_t column_in_tile = quarter * 32u + lane;
        const uint32_t lane_base = tmem_base + ((quarter * 32u) << 16) + group * S::kCols;
        uint32_t stage = 0, phase = 0, slot_phase = 0;
        bool ok = true;
        auto slot_ready = [&](uint32_t s, uint32_t parity) {
            // every lane waits (the wait does not consume the phase); the vote keeps the warp uniform
            const bool ready = __all_sync(0xffffffffu, wait_bounded_suspend(smem_u32(&control->slot_full[s]), parity,
                                                                            &control->abort_flag, p.error_word));
            fence_after();
            return ready;
        };
        uint32_t rbuf[2][kW];
        // the first block's first load
        if (blockIdx.x < tiles) {
            ok = slot_ready(0, 0);
            if (ok) tmem_ld<kW>(lane_base, rbuf[0]);
        }
        for (uint32_t tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
            const uint32_t m0 = (tile % p.m_tiles) * R + group * S::kCols;
            const uint32_t n_local = (tile / p.m_tiles) * kBW + column_in_tile;  // relative to col0
            const bool last_tile = tile + gridDim.x >= tiles;
            float acc[S::kCols];
#pragma unroll
            for (int j = 0; j < S::kCols; ++j) acc[j] = 0.0f;
            for (uint32_t ks = 0; ok && ks < p.k_stages; ++ks) {
                // this stage's scale boxes have landed
                ok = __all_sync(0xffffffffu, wait_bounded_suspend(smem_u32(&control->full[stage]), phase,
                                                                  &control->abort_flag, p.error_word));
                if (!ok) break;
                const float *scale_a = stage_da(stage) + group * S::kCols;
                const float *scale_w = stage_dw(stage) + column_in_tile;
                const bool more = ks + 1 < p.k_stages || !last_tile;
#pragma unroll
                for (int b = 0; b < kKB; ++b) {
                    const uint32_t taddr = lane_base + b * R;
                    const float dw = scale_w[b * kBW];
#pragma unroll
                    for (int c = 0; c < S::kChunks; ++c) {
                        const int t = b * S::kChunks + c;  // even: rbuf[0], odd: rbuf[1]
                        tmem_wait_ld<kW>(rbuf[t & 1]);
                        if (c + 1 < S::kChunks) {
                            tmem_ld<kW>(taddr + (c + 1) * kW, rbuf[(t + 1) & 1]);
                        } else {
                            fence_before();
                            mbar_arrive(smem_u32(&control->slot_empty[b]));  // this thread has read the slot
                            if (b + 1 < kKB) {
                                ok = slot_ready(b + 1, slot_phase);
                                if (ok) tmem_ld<kW>(taddr + R, rbuf[(t + 1) & 1]);
                            } else if (more) {
                                ok = slot_ready(0, slot_phase ^ 1u);
                                if (ok) tmem_ld<kW>(lane_base, rbuf[(t + 1) & 1]);
                            }
                        }
                        accumulate<kW>(acc + c * kW, rbuf[t & 1], scale_a + b * R + c * kW, dw);
                    }
                    if (!ok) break;
                }
                if (!ok) break;
                mbar_arrive(smem_u32(&control->empty[stage]));  // done with this stage's scales
                slot_phase ^= 1u;
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
            if (n_local < p.count) {
                float *out = p.destination + static_cast<size_t>(m0) * p.destination_stride + p.out_col0 + n_local;
#pragma unroll
                for (int j = 0; j < S::kCols; ++j)
                    if (m0 + j < p.rows) out[static_cast<size_t>(j) * p.destination_stride] = acc[j];
            }
        }
        if (!ok) tmem_wait_ld<kW>(rbuf[0]);  // a load issued before the abort lands before tensor memory is freed
    }

    fence_before();
    __syncthreads();
    if (warp == 1) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(S::kTmemCols) : "memory");
    }
}

// Native-to-MX weight expansion (prepare time): codes of [columns][blocks][16] nibble bytes to
// int8 (code - 8) rows of blocks_pad * 32 bytes (zero padding), fp16 scales [columns][scale_stride]
// to fp32 block-major [blocks_pad][columns] (zeros for padded blocks). One thread per (column, block).
__global__ void __launch_bounds__(256) q4_0_mx_expand_kernel(const uint8_t *__restrict__ nibbles,
                                                             const uint16_t *__restrict__ scales, uint32_t columns,
                                                             uint32_t blocks, uint32_t blocks_pad, uint32_t scale_stride,
                                                             int8_t *__restrict__ values, float *__restrict__ scales_t) {
    const uint64_t total = static_cast<uint64_t>(columns) * blocks_pad;
    for (uint64_t item = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; item < total;
         item += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t column = static_cast<uint32_t>(item / blocks_pad);
        const uint32_t block = static_cast<uint32_t>(item % blocks_pad);
        int8_t out[32] = {};
        float d = 0.0f;
        if (block < blocks) {
            // byte j of the block holds code j in its low nibble and code j + 16 in its high nibble
            const uint8_t *codes = nibbles + (static_cast<size_t>(column) * blocks + block) * 16;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                out[j] = static_cast<int8_t>(static_cast<int>(codes[j] & 0x0F) - 8);
                out[16 + j] = static_cast<int8_t>(static_cast<int>(codes[j] >> 4) - 8);
            }
            d = __half2float(__ushort_as_half(scales[static_cast<size_t>(column) * scale_stride + block]));
        }
        int8_t *row = values + (static_cast<size_t>(column) * blocks_pad + block) * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) row[j] = out[j];
        scales_t[static_cast<size_t>(block) * columns + column] = d;
    }
}

}  // namespace
}  // namespace qpucuda

namespace qpucuda {

bool q4_0_mx_sm100_available(int cc_major, int cc_minor) { return cc_major == 10 && cc_minor == 0; }

cudaError_t launch_q4_0_mx_expand(const uint8_t *nibbles, const uint16_t *scales, uint32_t columns, uint32_t blocks,
                                  uint32_t blocks_pad, uint32_t scale_stride, int8_t *values, float *scales_t,
                                  cudaStream_t stream) {
    const uint64_t items = static_cast<uint64_t>(columns) * blocks_pad;
    if (items == 0) return cudaSuccess;
    const uint32_t grid = static_cast<uint32_t>(items / 256 + 1 < 148ull * 32ull ? items / 256 + 1 : 148ull * 32ull);
    q4_0_mx_expand_kernel<<<grid, 256, 0, stream>>>(nibbles, scales, columns, blocks, blocks_pad, scale_stride, values,
                                                    scales_t);
    return cudaGetLastError();
}

namespace {

uint32_t mx_row_tile(uint32_t rows) { return rows <= 16 ? 16u : rows <= 32 ? 32u : rows <= 64 ? 64u : 128u; }

template <int R, int G>
cudaError_t launch_shape(const int8_t *q, const float *da_t, uint32_t rows, uint32_t rows_pad, const int8_t *values,
                         const float *scales_t, uint32_t columns, uint32_t blocks_pad, float *destination,
                         size_t destination_stride, uint32_t col0, uint32_t out_col0, uint32_t count,
                         unsigned int *error_word, int sm_count, cudaStream_t stream) {
    using S = MxShape<R, G>;
    constexpr size_t kSmem = smem_bytes<R, G>();
    static_assert(kSmem <= 227 * 1024, "shared memory budget");
    static PerDeviceOnce configured;
    const cudaError_t configure_error = configured.run([] {
        return cudaFuncSetAttribute(q4_0_mx_sm100_kernel<R, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(kSmem));
    });
    if (configure_error != cudaSuccess) return configure_error;
    const uint64_t k_bytes = static_cast<uint64_t>(blocks_pad) * 32;
    CUtensorMap map_a, map_w, map_da, map_dw;
    if (!encode_tensor_map_2d_u8(&map_a, q, k_bytes, rows_pad, k_bytes, 128, R) ||
        !encode_tensor_map_2d_u8(&map_w, values, k_bytes, columns, k_bytes, 128, kBW) ||
        !encode_tensor_map_2d_f32(&map_da, da_t, rows_pad, blocks_pad, static_cast<uint64_t>(rows_pad) * 4, R, kKB) ||
        !encode_tensor_map_2d_f32(&map_dw, scales_t, columns, blocks_pad, static_cast<uint64_t>(columns) * 4, kBW, kKB)) {
        return cudaErrorInvalidValue;
    }
    MxParams p{};
    p.rows = rows;
    p.k_stages = blocks_pad / kKB;
    p.m_tiles = (rows + R - 1) / R;
    p.n_tiles = (count + kBW - 1) / kBW;
    p.col0 = col0;
    p.count = count;
    p.out_col0 = out_col0;
    p.destination = destination;
    p.destination_stride = destination_stride;
    p.error_word = error_word;
    const uint64_t tiles = static_cast<uint64_t>(p.m_tiles) * p.n_tiles;
    const uint64_t slots = static_cast<uint64_t>(sm_count) * S::kCtasPerSm;
    const uint32_t grid = static_cast<uint32_t>(tiles < slots ? tiles : slots);
    q4_0_mx_sm100_kernel<R, G><<<grid, S::kThreads, kSmem, stream>>>(map_a, map_w, map_da, map_dw, p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_q4_0_mx_sm100(const int8_t *q, const float *da_t, uint32_t rows, uint32_t rows_pad,
                                 const int8_t *values, const float *scales_t, uint32_t columns, uint32_t blocks,
                                 uint32_t blocks_pad, float *destination, size_t destination_stride, uint32_t col0,
                                 uint32_t out_col0, uint32_t count, unsigned int *error_word, int sm_count,
                                 cudaStream_t stream) {
    if (rows == 0 || count == 0) return cudaSuccess;
    if (blocks_pad % kKB != 0 || blocks_pad < blocks || col0 % 16 != 0 || columns % 4 != 0 || rows_pad % 4 != 0 ||
        col0 + count > columns) {
        return cudaErrorInvalidValue;
    }
#define QPUCUDA_MX_SHAPE(R, G)                                                                                       \
    launch_shape<R, G>(q, da_t, rows, rows_pad, values, scales_t, columns, blocks_pad, destination, destination_stride, \
                       col0, out_col0, count, error_word, sm_count, stream)
    // The smallest row tile that holds the call's rows (no padded rows computed). Measured on the
    // 70B gate shape (8192 -> 28672, 1 x B200): 16 rows with 8 epilogue warps (8 rows per thread)
    // 91 us against 105 us with 16 warps (4 rows per thread).
    switch (mx_row_tile(rows)) {
        case 16: return QPUCUDA_MX_SHAPE(16, 2);
        case 32: return QPUCUDA_MX_SHAPE(32, 2);
        case 64: return QPUCUDA_MX_SHAPE(64, 4);
        default: return QPUCUDA_MX_SHAPE(128, 4);
    }
#undef QPUCUDA_MX_SHAPE
}

bool q4_0_mx_sm100_fills_wave(uint32_t rows, uint32_t count, int sm_count) {
    const uint32_t r = mx_row_tile(rows);
    const uint64_t tiles = static_cast<uint64_t>((rows + r - 1) / r) * ((count + kBW - 1) / kBW);
    return tiles >= static_cast<uint64_t>(sm_count > 0 ? sm_count : 1);
}

}  // namespace qpucuda
