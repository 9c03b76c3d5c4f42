// W8A8 GEMM for sm_100a: int8 x int8 -> int32 on the 5th-generation tensor cores
// (tcgen05.mma kind::i8), operands staged by TMA, accumulators in tensor memory,
// fused dequant (+bias) epilogue.
//
// Replaces the reference's vc7.tiled_w8a8_gemm[_dequantize] QPU program
// (src/qpu_xla/kernels/gemm_int8.py:43-204): same contract, acc[m, n] =
// sum_k a[m, k] * w[n, k] exactly in int32, and, in the dequantize modes,
// out = ((float)acc * row_scale[m]) * col_scale[n] (gemm_int8.py:166-184,
// itof then two fmul in that order) with the bias added afterwards
// (src/qpu_xla/models/smolvla/accelerated.py:260-261). The epilogue uses
// __int2float_rn / __fmul_rn / __fadd_rn so nothing is contracted into an FMA
// and the result is bit-identical to the reference's NumPy arithmetic.
//
// Structure: one persistent CTA per SM (192 threads, ~225 KB of shared memory,
// so exactly one CTA per SM and its 512 TMEM columns are always free).
//   warp 0      TMA producer: A tile 128 x 128 B and W tile 256 x 128 B (two 128-row boxes)
//               per stage, 4-stage ring, 128-byte swizzle, mbarrier complete_tx.
//   warp 1      TMEM allocator and MMA issuer (one thread runs the loop): 4 x tcgen05.mma
//               (M=128, N=256, K=32) per stage; tcgen05.commit releases the stage and,
//               after the last K block, signals the accumulator buffer full.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns at a time, dequantize,
//               store; two accumulator buffers (2 x 256 columns) let the epilogue
//               of tile i overlap the main loop of tile i+1.
// Every mbarrier wait is bounded (globaltimer); on expiry the kernel records
// kKernelWaitTimeout in the error word, drains its own copies and MMAs with
// bounded waits, frees TMEM and returns. No multicast load is used anywhere.
//
// CTA-pair mode (PAIR, clusters of 2, tcgen05 cta_group::2): a 256 x 256 tile per pair; each CTA
// stages its 128 rows of A and 128 of the 256 W rows (256 bytes of K per stage, 64 KB, 3 stages)
// with TMA loads whose bytes complete on the leader (rank 0) CTA's barrier; the leader issues
// M = 256 MMAs that read both CTAs' shared memory and write each CTA's 128 accumulator rows into
// its own tensor memory; its commits arrive on the stage and accumulator barriers of both CTAs; each CTA's
// epilogue drains its own rows and releases the buffer on the leader's barrier. The protocol
// (who arms which barrier, the same warp allocating tensor memory in both CTAs) follows
// CUTLASS's sm100 2-SM GEMM pipeline.
#include <cstring>

#include "qpucuda_internal.h"
#include "sm100_sync.cuh"

namespace qpucuda {
namespace {

constexpr int BM = 128;  // rows of A per CTA
constexpr int BN = 256;  // output columns per tile
constexpr int BK = 128;  // bytes (int8 elements) of K per stage = one 128-byte swizzle row
constexpr int UMMA_K = 32;  // K per tcgen05.mma kind::i8
constexpr int TMEM_COLS = 2 * BN;  // two s32 accumulators of BN columns
constexpr int NUM_THREADS = 192;
constexpr int EPILOGUE_THREADS = 128;
constexpr int W_BOX_ROWS = 128;  // rows of W per TMA box (a 256-row B tile is two boxes)

// Pipeline shape per mode. Single-CTA: A 128 x 128 B + B 256 x 128 B = 48 KB per stage, 4 stages.
// CTA pair (tcgen05 cta_group::2, M = 256 across two SMs): each CTA stages its own 128 rows of A
// and its half (128 rows) of B for 256 bytes of K, 64 KB per stage, 3 stages.
template <bool PAIR>
struct Pipe {
    // 128-byte K boxes per stage and per operand: CTA pairs take two (256 bytes of K, eight
    // MMAs between barrier round trips)
    static constexpr int K_BOXES = PAIR ? 2 : 1;
    static constexpr int STAGES = PAIR ? 3 : 4;
    static constexpr int A_BOX_BYTES = BM * BK;
    static constexpr int B_BOX_BYTES = (PAIR ? BN / 2 : BN) * BK;
    static constexpr int A_BYTES = K_BOXES * A_BOX_BYTES;
    static constexpr int B_BYTES = K_BOXES * B_BOX_BYTES;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int K_STAGE = K_BOXES * BK;  // bytes of K per stage
};

static_assert(BN == kGemmBlockN && BM == kGemmBlockM && BK == kGemmBlockK && W_BOX_ROWS == kGemmWeightBoxRows,
              "tile constants must agree");

// Instruction descriptor (kind::i8): D = s32 (bits 4-5 = 2), A = s8 (bits 7-9 = 1),
// B = s8 (bits 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bits 17-22,
// M >> 4 at bits 24-28.
constexpr uint32_t kInstrDesc = (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
                                (static_cast<uint32_t>(BM >> 4) << 24);
// The same for the CTA pair: M = 256 (each CTA's tensor memory receives its 128 rows).
constexpr uint32_t kInstrDescPair = (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
                                    (static_cast<uint32_t>((2 * BM) >> 4) << 24);

template <int NSTAGES>
struct Control {
    uint64_t full[NSTAGES];
    uint64_t empty[NSTAGES];
    uint64_t tmem_full[2];
    uint64_t tmem_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    volatile int abort_flag;
};

// Epilogue staging, 8 KB per epilogue warp: two 4 KB buffers of 32 rows x 128 bytes (128-byte
// swizzle) that TMA stores copy to the output, or, with peer destinations, the 4 KB transpose
// buffer that turns each lane's row values into 128-byte row segments for plain stores.
constexpr int EPILOGUE_WARP_BYTES = 8192;
constexpr int EPILOGUE_STAGE_BYTES = (EPILOGUE_THREADS / 32) * EPILOGUE_WARP_BYTES;
template <bool PAIR>
constexpr size_t smem_bytes() {
    return static_cast<size_t>(Pipe<PAIR>::STAGES) * Pipe<PAIR>::STAGE_BYTES + EPILOGUE_STAGE_BYTES + 1024 +
           sizeof(Control<Pipe<PAIR>::STAGES>);
}
static_assert(smem_bytes<false>() <= 227 * 1024 && smem_bytes<true>() <= 227 * 1024, "shared memory budget");

struct GemmParams {
    uint32_t m, n, k;
    uint32_t num_kb;
    uint32_t m_blocks, n_blocks;
    int mode;
    const float *row_scales;
    const float *col_scales;
    const float *bias;
    void *out;
    size_t out_stride;
    // Further destinations written with the same (row, column) offsets and row stride as
    // `out`: other ranks' output buffers for the fused GEMM + all-gather.
    void *peer_out[kGemmMaxPeers];
    uint32_t peer_count;
    // Output (m, n) at (m / rows_per_batch) * batch_stride + (m % rows_per_batch) * out_stride
    // + n * col_stride elements (row-major: rows_per_batch >= m, col_stride 1).
    uint32_t rows_per_batch;
    size_t batch_stride;
    size_t col_stride;
    // Local row-major output written by TMA stores through map_out (32 x 32 boxes).
    uint32_t tma_store;
    unsigned int *error_word;
    // Split-K (single-CTA tiles, int32 output only): work unit u is tile u % tiles over K stages
    // [s * kb_per_split, (s + 1) * kb_per_split) with s = u / tiles; its rows go to output rows
    // s * split_rows + m (split_rows a multiple of the tile rows). splits = 1: no split.
    uint32_t splits;
    uint32_t kb_per_split;
    uint32_t split_rows;
    uint32_t group_rows;  // row blocks per tile group (see tile_coords)
};

using namespace sm100;

// Tile order: groups of group_rows row blocks, and within a group the row block fastest. The
// CTAs (pairs) resident at once then cover a few column blocks of every row block of the group,
// so the group's A rows stay in L2 while its columns stream past, and each W tile is read from
// DRAM once per group. A row-fastest order over all row blocks re-read the whole A from DRAM on
// every wave once A outgrew L2 (the 70B down projection's 117 MB A was read 7 times). The host
// takes as many row blocks per group as keep the group's A within ~40 MB, at least 8: every row
// block of the 70B gate and up (16 blocks of 2 MB, so W is read once), 8 for the down projection.
constexpr uint32_t kTileGroupRows = 8;
constexpr uint64_t kTileGroupBytes = 40ull << 20;
__device__ __forceinline__ void tile_coords(uint32_t tile, uint32_t m_blocks, uint32_t n_blocks, uint32_t &m_block,
                                            uint32_t &n_block, uint32_t group_rows) {
    const uint32_t group_tiles = group_rows * n_blocks;
    const uint32_t group = tile / group_tiles;
    const uint32_t first = group * group_rows;
    const uint32_t rows = min(group_rows, m_blocks - first);
    const uint32_t local = tile - group * group_tiles;
    m_block = first + local % rows;
    n_block = local / rows;
}

// Bounded wait on this CTA's abort flag (see sm100_sync.cuh).
template <int NSTAGES>
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, Control<NSTAGES> *control,
                                             unsigned int *error_word) {
    return sm100::wait_bounded(bar, parity, &control->abort_flag, error_word);
}

// ---- CTA-pair (cluster of 2) primitives, in the forms CUTLASS's sm100 2-SM GEMM uses ----
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t rank;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    return rank;
}
// Address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t address, uint32_t rank) {
    uint32_t mapped;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(mapped) : "r"(address), "r"(rank));
    return mapped;
}
__device__ __forceinline__ void remote_arrive(uint32_t cluster_address) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_address) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}
// 2D tiled TMA load into this CTA's shared memory whose bytes complete on the leader CTA's
// mbarrier (cta_group::2 form; no multicast).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t destination, const CUtensorMap *map, uint32_t leader_bar,
                                                 int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(destination),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y)
        : "memory");
}

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle
// canonical layout: rows of 128 bytes, 8-row (1024-byte) swizzle atoms stacked
// along M/N. start >> 4 at bits 0-13, LBO = 16 B (unused for swizzled K-major)
// at 16-29, SBO = 1024 B at 32-45, descriptor version 1 at bit 46, layout
// SWIZZLE_128B (2) at bits 61-63.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t address) {
    uint64_t desc = static_cast<uint64_t>((address & 0x3FFFFu) >> 4);
    desc |= static_cast<uint64_t>(1) << 16;
    desc |= static_cast<uint64_t>(1024 >> 4) << 32;
    desc |= static_cast<uint64_t>(1) << 46;
    desc |= static_cast<uint64_t>(2) << 61;
    return desc;
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(kInstrDesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// CTA pair: one MMA over both CTAs' operands (same shared-memory offsets in each), writing each
// CTA's 128 rows into its own tensor memory.
__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(kInstrDescPair), "r"(accumulate)
        : "memory");
}
// Completion of the pair's MMAs signalled on the barrier at `bar`'s offset in both CTAs.
__device__ __forceinline__ void umma_commit_pair_both(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 ::"r"(bar), "h"(static_cast<uint16_t>(3))
                 : "memory");
}
// ... on this CTA's barrier only (abort drain).
__device__ __forceinline__ void umma_commit_pair_local(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_load_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// TMA store of a 32-row x 128-byte box from this CTA's shared memory (bulk async group).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t source, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(source), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// All but the newest bulk group have finished reading their shared-memory source.
__device__ __forceinline__ void bulk_wait_read_all_but_one() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Generic-proxy shared-memory writes made visible to the async proxy (TMA).
__device__ __forceinline__ void fence_proxy_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ float dequant(uint32_t bits, float row_scale, float col_scale) {
    return __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(bits)), row_scale), col_scale);
}

// Packed fp32 pairs (sm_100 mul.f32x2 with explicit round-to-nearest): each half rounds exactly
// as __fmul_rn, two values per instruction.
__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
    return static_cast<unsigned long long>(__float_as_uint(lo)) | (static_cast<unsigned long long>(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// One row's 32 accumulators of columns n0 .. n0 + 31 (all in range), dequantized in place:
// ((float)acc * row_scale) * col_scale[n] (+ bias[n]) in that order, the scales and bias read
// with one 16-byte load per four columns (every lane reads the same address). `cs` and `cb` are
// 16-byte aligned.
template <bool BIAS>
__device__ __forceinline__ void dequant_chunk_vec(uint32_t (&r)[32], float row_scale, const float *cs, const float *cb) {
    const unsigned long long row2 = pack2(row_scale, row_scale);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const float4 c = __ldg(reinterpret_cast<const float4 *>(cs) + q);
        unsigned long long lo = pack2(__int2float_rn(static_cast<int>(r[4 * q])), __int2float_rn(static_cast<int>(r[4 * q + 1])));
        unsigned long long hi = pack2(__int2float_rn(static_cast<int>(r[4 * q + 2])), __int2float_rn(static_cast<int>(r[4 * q + 3])));
        lo = mul2(mul2(lo, row2), pack2(c.x, c.y));
        hi = mul2(mul2(hi, row2), pack2(c.z, c.w));
        float v0 = __uint_as_float(static_cast<uint32_t>(lo)), v1 = __uint_as_float(static_cast<uint32_t>(lo >> 32));
        float v2 = __uint_as_float(static_cast<uint32_t>(hi)), v3 = __uint_as_float(static_cast<uint32_t>(hi >> 32));
        if constexpr (BIAS) {
            const float4 b = __ldg(reinterpret_cast<const float4 *>(cb) + q);
            v0 = __fadd_rn(v0, b.x);
            v1 = __fadd_rn(v1, b.y);
            v2 = __fadd_rn(v2, b.z);
            v3 = __fadd_rn(v3, b.w);
        }
        r[4 * q] = __float_as_uint(v0);
        r[4 * q + 1] = __float_as_uint(v1);
        r[4 * q + 2] = __float_as_uint(v2);
        r[4 * q + 3] = __float_as_uint(v3);
    }
}

// The same for a chunk with `valid` (< 32) columns in range, or unaligned scales: scalar loads
// (every lane reads the same address), zeros past the last column.
__device__ __forceinline__ void dequant_chunk_scalar(uint32_t (&r)[32], float row_scale, const float *cs, const float *cb,
                                                     bool with_bias, uint32_t valid) {
#pragma unroll
    for (uint32_t j = 0; j < 32; ++j) {
        const bool in_range = j < valid;
        float v = dequant(r[j], row_scale, in_range ? __ldg(cs + j) : 0.0f);
        if (with_bias) v = __fadd_rn(v, in_range ? __ldg(cb + j) : 0.0f);
        r[j] = __float_as_uint(v);
    }
}

__device__ __forceinline__ void dequant_chunk(uint32_t (&r)[32], float row_scale, const float *cs, const float *cb,
                                              bool with_bias, uint32_t valid, bool vector_scales) {
    if (valid >= 32 && vector_scales) {
        if (with_bias) {
            dequant_chunk_vec<true>(r, row_scale, cs, cb);
        } else {
            dequant_chunk_vec<false>(r, row_scale, cs, cb);
        }
    } else {
        dequant_chunk_scalar(r, row_scale, cs, cb, with_bias, valid);
    }
}

// Four consecutive 4-byte outputs of one row, columns col..col+3 (the caller guarantees
// col < n); a 16-byte store when the whole group is in range and aligned.
__device__ __forceinline__ void store_group(void *base, size_t offset, uint4 value, uint32_t valid, bool aligned) {
    uint32_t *p = static_cast<uint32_t *>(base) + offset;
    if (valid >= 4 && aligned) {
        *reinterpret_cast<uint4 *>(p) = value;
        return;
    }
    p[0] = value.x;
    if (valid > 1) p[1] = value.y;
    if (valid > 2) p[2] = value.z;
    if (valid > 3) p[3] = value.w;
}

// FANOUT: the epilogue also writes every peer destination (fused GEMM + all-gather).
// PAIR: launched as clusters of two CTAs that share each 256-row tile (tcgen05 cta_group::2):
// CTA rank r loads rows r*128.. of the tile's A rows and of its 256 W rows; the rank-0 (leader)
// CTA issues the MMAs for both and each CTA's epilogue drains its own 128 rows. Tiles are then
// 256 x 256 per pair and params.m_blocks counts 256-row blocks.
template <bool FANOUT, bool PAIR>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    w8a8_gemm_sm100_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                           const __grid_constant__ CUtensorMap map_out, const GemmParams params) {
    constexpr int STAGES = Pipe<PAIR>::STAGES;
    constexpr int A_STAGE_BYTES = Pipe<PAIR>::A_BYTES;
    constexpr int B_STAGE_BYTES = Pipe<PAIR>::B_BYTES;
    constexpr int STAGE_BYTES = Pipe<PAIR>::STAGE_BYTES;
    using Control = qpucuda::Control<STAGES>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *stage_a = smem;
    uint8_t *stage_b = smem + STAGES * A_STAGE_BYTES;
    uint4 *epilogue_stage = reinterpret_cast<uint4 *>(smem + STAGES * STAGE_BYTES);
    Control *control = reinterpret_cast<Control *>(smem + STAGES * STAGE_BYTES + EPILOGUE_STAGE_BYTES);

    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t num_tiles = params.m_blocks * params.n_blocks;
    const uint32_t num_units = num_tiles * params.splits;  // (tile, K slice) pairs
    auto unit_range = [&](uint32_t unit, uint32_t &tile, uint32_t &kb_begin, uint32_t &kb_end) {
        tile = unit % num_tiles;
        kb_begin = (unit / num_tiles) * params.kb_per_split;
        kb_end = min(params.num_kb, kb_begin + params.kb_per_split);
    };
    const uint32_t rank = PAIR ? cluster_rank() : 0u;  // this CTA's half of the pair
    const bool leader = rank == 0;
    const uint32_t first_tile = PAIR ? blockIdx.x / 2 : blockIdx.x;
    const uint32_t tile_step = PAIR ? gridDim.x / 2 : gridDim.x;
    constexpr uint32_t kTileRows = PAIR ? 2 * BM : BM;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&control->full[s]), 1);
            mbar_init(smem_u32(&control->empty[s]), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_u32(&control->tmem_full[i]), 1);
            // the leader's MMA waits for the epilogue warps of both CTAs
            mbar_init(smem_u32(&control->tmem_empty[i]), (PAIR ? 2 : 1) * EPILOGUE_THREADS / 32);
        }
        mbar_init(smem_u32(&control->drain), 1);
        control->abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        // CTA pair: the same warp of both CTAs allocates collectively, into the same offset.
        if constexpr (PAIR) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32(&control->tmem_base)),
                         "r"(TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32(&control->tmem_base)),
                         "r"(TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync();  // both CTAs' barriers exist before any remote arrive or copy
    tc_fence_after();
    const uint32_t tmem_base = control->tmem_base;
    // Programmatic dependent launch: the set-up above (barriers, tensor memory) overlaps the end of
    // the previous kernel on the stream (the row quantizer, whose output this kernel reads); every
    // global read and write below comes after the wait. The next kernel may launch at once: it
    // waits for this grid in turn before touching memory.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            prefetch_tensor_map(&map_a);
            prefetch_tensor_map(&map_w);
            uint32_t stage = 0, phase = 0;
            // Per stage (bit s): a copy was issued on it, and the phase it was issued in. Bit masks
            // rather than arrays indexed by the runtime stage, which would live in local memory.
            uint32_t issued_mask = 0, issued_phases = 0;
            bool ok = true;
            for (uint32_t unit = first_tile; ok && unit < num_units; unit += tile_step) {
                uint32_t tile, kb_begin, kb_end;
                unit_range(unit, tile, kb_begin, kb_end);
                uint32_t m_block, n_block;
                tile_coords(tile, params.m_blocks, params.n_blocks, m_block, n_block, params.group_rows);
                const int m0 = static_cast<int>(m_block * kTileRows + rank * BM);
                const int n0 = static_cast<int>(n_block * BN);
                for (uint32_t kb = kb_begin; kb < kb_end; ++kb) {
                    if (!wait_bounded(smem_u32(&control->empty[stage]), phase ^ 1u, control, params.error_word)) {
                        ok = false;
                        break;
                    }
                    const uint32_t full = smem_u32(&control->full[stage]);
                    const int x = static_cast<int>(kb * Pipe<PAIR>::K_STAGE);
                    if constexpr (PAIR) {
                        // Both CTAs' bytes complete on the leader's barrier, which expects them all.
                        if (leader) mbar_expect_tx(full, 2 * STAGE_BYTES);
                        const uint32_t leader_full = map_to_rank(full, 0);
#pragma unroll
                        for (int box = 0; box < Pipe<PAIR>::K_BOXES; ++box) {
                            tma_load_2d_pair(smem_u32(stage_a + stage * A_STAGE_BYTES + box * Pipe<PAIR>::A_BOX_BYTES),
                                             &map_a, leader_full, x + box * BK, m0);
                            tma_load_2d_pair(smem_u32(stage_b + stage * B_STAGE_BYTES + box * Pipe<PAIR>::B_BOX_BYTES),
                                             &map_w, leader_full, x + box * BK, n0 + static_cast<int>(rank) * W_BOX_ROWS);
                        }
                    } else {
                        mbar_expect_tx(full, STAGE_BYTES);
                        tma_load_2d(smem_u32(stage_a + stage * A_STAGE_BYTES), &map_a, full, x, m0);
                        tma_load_2d(smem_u32(stage_b + stage * B_STAGE_BYTES), &map_w, full, x, n0);
                        tma_load_2d(smem_u32(stage_b + stage * B_STAGE_BYTES + W_BOX_ROWS * BK), &map_w, full, x,
                                    n0 + W_BOX_ROWS);
                    }
                    issued_mask |= 1u << stage;
                    issued_phases = (issued_phases & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                // Abort path: let every copy this thread started land before the CTA exits. In a
                // pair only the leader's barriers see the copies (of both CTAs); the other CTA
                // gives its copies in flight a bounded 200 us instead.
                if (!PAIR || leader) {
                    for (int s = 0; s < STAGES; ++s) {
                        if ((issued_mask >> s) & 1u) wait_drain(smem_u32(&control->full[s]), (issued_phases >> s) & 1u);
                    }
                } else {
                    const uint64_t start = globaltimer();
                    while (globaltimer() - start < 200000ull) {
                    }
                }
            }
        }
        __syncwarp();  // reconverge before the CTA barrier at the end
    } else if (warp == 1) {
        // ---------------- MMA issuer (the leader CTA only, in a pair) ----------------
        // One thread runs the whole loop: it waits on the barriers, fences and issues; the warp's
        // other lanes wait at the final __syncwarp.
        if (lane == 0 && (!PAIR || leader)) {
            uint32_t stage = 0, phase = 0, local_tile = 0;
            bool ok = true, any_mma = false;
            for (uint32_t unit = first_tile; ok && unit < num_units; unit += tile_step, ++local_tile) {
                uint32_t tile, kb_begin, kb_end;
                unit_range(unit, tile, kb_begin, kb_end);
                const uint32_t acc = local_tile & 1u;
                const uint32_t acc_phase = (local_tile >> 1) & 1u;
                ok = wait_bounded(smem_u32(&control->tmem_empty[acc]), acc_phase ^ 1u, control, params.error_word);
                if (!ok) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (uint32_t kb = kb_begin; kb < kb_end; ++kb) {
                    ok = wait_bounded(smem_u32(&control->full[stage]), phase, control, params.error_word);
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < Pipe<PAIR>::K_STAGE / UMMA_K; ++kk) {
                        // box kk / 4 of the stage; within it, the start address advances by 32 bytes
                        // (encoded >> 4) along the swizzle row
                        constexpr int kPerBox = BK / UMMA_K;
                        const int box = kk / kPerBox;
                        const uint64_t a = smem_desc_sw128(smem_u32(stage_a + stage * A_STAGE_BYTES + box * Pipe<PAIR>::A_BOX_BYTES)) +
                                           static_cast<uint64_t>((kk % kPerBox) * (UMMA_K >> 4));
                        const uint64_t b = smem_desc_sw128(smem_u32(stage_b + stage * B_STAGE_BYTES + box * Pipe<PAIR>::B_BOX_BYTES)) +
                                           static_cast<uint64_t>((kk % kPerBox) * (UMMA_K >> 4));
                        if constexpr (PAIR) {
                            umma_i8_pair(d_tmem, a, b, (kb != kb_begin || kk != 0) ? 1u : 0u);
                        } else {
                            umma_i8(d_tmem, a, b, (kb != kb_begin || kk != 0) ? 1u : 0u);
                        }
                    }
                    // frees this stage in both CTAs of a pair
                    if constexpr (PAIR) {
                        umma_commit_pair_both(smem_u32(&control->empty[stage]));
                    } else {
                        umma_commit(smem_u32(&control->empty[stage]));
                    }
                    any_mma = true;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                if constexpr (PAIR) {
                    umma_commit_pair_both(smem_u32(&control->tmem_full[acc]));
                } else {
                    umma_commit(smem_u32(&control->tmem_full[acc]));
                }
            }
            if (!ok && any_mma) {
                // Abort path: wait for every MMA this thread issued before TMEM is freed.
                if constexpr (PAIR) {
                    umma_commit_pair_local(smem_u32(&control->drain));
                } else {
                    umma_commit(smem_u32(&control->drain));
                }
                wait_drain(smem_u32(&control->drain), 0);
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        // Lane l of warp w reads TMEM lane (w % 4) * 32 + l, i.e. one output row, 32 columns per
        // tcgen05.ld, and converts the values in registers. A local row-major output is stored
        // straight from registers. With peer destinations the values are written to this warp's
        // 4 KB staging buffer as 8 x 16 bytes per row (16-byte slot c of row r at c ^ (r & 7):
        // conflict-free both ways) and read back row-wise: 8 lanes cover one row's 32 columns,
        // so each store instruction writes four 128-byte row segments, to `out` and to every
        // peer (full-line writes over NVLink).
        const uint32_t quarter = warp & 3u;  // TMEM lanes this warp may access
        uint4 *staging = epilogue_stage + (warp - 2u) * (EPILOGUE_WARP_BYTES / 16);
        const bool tma_store = !FANOUT && params.tma_store != 0;
        uint32_t stores_issued = 0;  // bulk groups this warp committed (selects the staging buffer)
        if (tma_store && lane == 0) prefetch_tensor_map(&map_out);
        const bool s32 = params.mode == static_cast<int>(EpilogueMode::kStoreS32);
        const bool with_bias = params.mode == static_cast<int>(EpilogueMode::kDequantizeBias);
        // Column scales and bias in 16-byte loads (chunks start at multiples of 32 columns).
        const bool vector_scales = (reinterpret_cast<uintptr_t>(params.col_scales) & 15u) == 0 &&
                                   (!with_bias || (reinterpret_cast<uintptr_t>(params.bias) & 15u) == 0);
        // Row-segment stores need unit column stride; otherwise (NCHW outputs) each lane stores its
        // own row's values straight from registers, which is coalesced when rows are adjacent.
        const bool row_segments = params.col_stride == 1;
        // Batched rows (NCHW outputs) need a division per row; plain row-major outputs do not.
        const bool batched = params.rows_per_batch != 0xFFFFFFFFu;
        const uint32_t peers = FANOUT ? params.peer_count : 0u;
        bool aligned = (params.out_stride & 3u) == 0 && (params.batch_stride & 3u) == 0 &&
                       (reinterpret_cast<uintptr_t>(params.out) & 15u) == 0;
        if constexpr (FANOUT) {
#pragma unroll
            for (uint32_t d = 0; d < kGemmMaxPeers; ++d)
                if (d < peers) aligned = aligned && (reinterpret_cast<uintptr_t>(params.peer_out[d]) & 15u) == 0;
        }
        // Release of an accumulator buffer goes to the MMA issuer's barrier (the leader's in a pair).
        const uint32_t empty_bar0 = PAIR ? map_to_rank(smem_u32(&control->tmem_empty[0]), 0) : smem_u32(&control->tmem_empty[0]);
        const uint32_t empty_bar1 = PAIR ? map_to_rank(smem_u32(&control->tmem_empty[1]), 0) : smem_u32(&control->tmem_empty[1]);
        uint32_t local_tile = 0;
        for (uint32_t unit = first_tile; unit < num_units; unit += tile_step, ++local_tile) {
            uint32_t tile, kb_begin, kb_end;
            unit_range(unit, tile, kb_begin, kb_end);
            const uint32_t split_row0 = (unit / num_tiles) * params.split_rows;  // 0 without a split
            const uint32_t acc = local_tile & 1u;
            const uint32_t acc_phase = (local_tile >> 1) & 1u;
            uint32_t m_block, n_block;
            tile_coords(tile, params.m_blocks, params.n_blocks, m_block, n_block, params.group_rows);
            const uint32_t n_base = n_block * BN;
            bool ok = true;
            if (lane == 0) ok = wait_bounded(smem_u32(&control->tmem_full[acc]), acc_phase, control, params.error_word);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            tc_fence_after();

            const uint32_t row0 = m_block * kTileRows + rank * BM + quarter * 32;  // first row of this warp
            const uint32_t m = row0 + lane;
            const float row_scale = (m < params.m && !s32) ? params.row_scales[m] : 0.0f;
            const size_t row_base = batched ? static_cast<size_t>(m / params.rows_per_batch) * params.batch_stride +
                                                  static_cast<size_t>(m % params.rows_per_batch) * params.out_stride
                                            : static_cast<size_t>(m) * params.out_stride;
            const uint32_t taddr = tmem_base + ((quarter * 32u) << 16) + acc * BN;
#pragma unroll 1
            for (uint32_t chunk = 0; chunk < BN / 32; ++chunk) {
                uint32_t r[32];
                tmem_load_32x32b_x32(taddr + chunk * 32, r);
                const uint32_t n0 = n_base + chunk * 32;
                if (n0 >= params.n) continue;  // warp-uniform
                const bool full_chunk = n0 + 32 <= params.n;
                if (tma_store) {
                    // Rows past m and columns past n fall outside the tensor map and are not written.
                    if (row0 >= params.m) continue;  // warp-uniform
                    if (!s32) {
                        dequant_chunk(r, row_scale, params.col_scales + n0, params.bias + n0, with_bias,
                                      full_chunk ? 32u : params.n - n0, vector_scales);
                    }
                    uint4 *buffer = staging + (stores_issued & 1u) * 256u;
                    if (lane == 0) bulk_wait_read_all_but_one();  // the store from this buffer has read it
                    __syncwarp();
#pragma unroll
                    for (uint32_t c = 0; c < 8; ++c)
                        buffer[lane * 8u + (c ^ (lane & 7u))] =
                            make_uint4(r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
                    fence_proxy_async_shared();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&map_out, smem_u32(buffer), static_cast<int>(n0), static_cast<int>(split_row0 + row0));
                        bulk_commit();
                    }
                    ++stores_issued;
                    continue;
                }
                if (!FANOUT && row_segments) {
                    // Local row-major output: each lane converts and stores its own row's 32 values
                    // as eight 16-byte stores (measured faster than a shared-memory transpose when
                    // nothing crosses NVLink).
                    if (m >= params.m) continue;
                    if (s32) {
                        int32_t *row = static_cast<int32_t *>(params.out) + row_base + n0;
                        if (full_chunk && (reinterpret_cast<uintptr_t>(row) & 15u) == 0) {
#pragma unroll
                            for (int j = 0; j < 32; j += 4)
                                *reinterpret_cast<int4 *>(row + j) =
                                    make_int4(static_cast<int>(r[j]), static_cast<int>(r[j + 1]), static_cast<int>(r[j + 2]),
                                              static_cast<int>(r[j + 3]));
                        } else {
                            // fully unrolled: r stays in registers (a runtime-bounded index would
                            // move the whole array to local memory)
#pragma unroll
                            for (uint32_t j = 0; j < 32; ++j)
                                if (n0 + j < params.n) row[j] = static_cast<int>(r[j]);
                        }
                    } else {
                        // Column scales / bias: every lane reads the same address (an L1 broadcast).
                        const float *cs = params.col_scales + n0;
                        const float *cb = params.bias + n0;
                        float *row = static_cast<float *>(params.out) + row_base + n0;
                        if (full_chunk && (reinterpret_cast<uintptr_t>(row) & 15u) == 0) {
                            dequant_chunk(r, row_scale, cs, cb, with_bias, 32u, vector_scales);
#pragma unroll
                            for (int j = 0; j < 32; j += 4)
                                *reinterpret_cast<uint4 *>(row + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
                        } else {
                            const uint32_t valid = full_chunk ? 32u : params.n - n0;
                            dequant_chunk(r, row_scale, cs, cb, with_bias, valid, vector_scales);
#pragma unroll
                            for (uint32_t j = 0; j < 32; ++j)
                                if (j < valid) row[j] = __uint_as_float(r[j]);
                        }
                    }
                    continue;
                }
                if (!s32) {
                    dequant_chunk(r, row_scale, params.col_scales + n0, params.bias + n0, with_bias,
                                  full_chunk ? 32u : params.n - n0, vector_scales);
                }
                if (!row_segments) {
                    // Column-strided (NCHW) output: each lane stores its own row's values element by
                    // element; adjacent lanes (adjacent pixels) write adjacent addresses.
                    if (m < params.m) {
                        {
#pragma unroll
                            for (uint32_t j = 0; j < 32; ++j) {
                                if (n0 + j < params.n) {
                                    const size_t offset = row_base + static_cast<size_t>(n0 + j) * params.col_stride;
                                    static_cast<uint32_t *>(params.out)[offset] = r[j];
                                    if constexpr (FANOUT) {
#pragma unroll
                                        for (uint32_t d = 0; d < kGemmMaxPeers; ++d)
                                            if (d < peers) static_cast<uint32_t *>(params.peer_out[d])[offset] = r[j];
                                    }
                                }
                            }
                        }
                    }
                    continue;
                }
                // Fan-out, row-major: transpose through shared memory so that every store
                // instruction writes four full 128-byte row segments, locally and to each peer.
#pragma unroll
                for (uint32_t c = 0; c < 8; ++c)
                    staging[lane * 8u + (c ^ (lane & 7u))] = make_uint4(r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
                __syncwarp();
                const uint32_t c = lane & 7u;
                const uint32_t col = n0 + c * 4u;
#pragma unroll
                for (uint32_t k = 0; k < 8; ++k) {
                    const uint32_t i = k * 4u + (lane >> 3);
                    const uint4 value = staging[i * 8u + (c ^ (i & 7u))];
                    const uint32_t row = row0 + i;
                    if (row < params.m && col < params.n) {
                        const size_t offset =
                            (batched ? static_cast<size_t>(row / params.rows_per_batch) * params.batch_stride +
                                           static_cast<size_t>(row % params.rows_per_batch) * params.out_stride
                                     : static_cast<size_t>(row) * params.out_stride) +
                            col;
                        const uint32_t valid = params.n - col;
                        store_group(params.out, offset, value, valid, aligned);
#pragma unroll
                        for (uint32_t d = 0; d < kGemmMaxPeers; ++d)
                            if (d < peers) store_group(params.peer_out[d], offset, value, valid, aligned);
                    }
                }
                __syncwarp();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (PAIR) {
                    remote_arrive(acc == 0 ? empty_bar0 : empty_bar1);
                } else {
                    mbar_arrive(acc == 0 ? empty_bar0 : empty_bar1);
                }
            }
        }
        // TMA stores: complete before the CTA exits.
        if (tma_store && lane == 0) bulk_wait_all();
        __syncwarp();
        // Peer destinations: make this thread's remote stores visible system-wide before exit.
        if (FANOUT && params.peer_count != 0) __threadfence_system();
    }

    tc_fence_before();
    __syncthreads();
    // A pair finishes together: neither CTA exits (or frees tensor memory) while the other may
    // still read its shared memory, signal its barriers or write its tensor memory.
    if constexpr (PAIR) cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR) {
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                         : "memory");
        } else {
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                         : "memory");
        }
    }
}

}  // namespace

namespace {

template <bool FANOUT, bool PAIR>
cudaError_t configure_kernel() {
    return cudaFuncSetAttribute(w8a8_gemm_sm100_kernel<FANOUT, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem_bytes<PAIR>()));
}

// Clusters of two that can be resident at once (one CTA per SM), cached per device.
int resident_pairs(int sm_count) {
    static std::atomic<int> cached[64] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return sm_count / 2;
    const int known = cached[device].load(std::memory_order_relaxed);
    if (known > 0) return known;
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(static_cast<unsigned>(sm_count & ~1), 1, 1);
    config.blockDim = dim3(NUM_THREADS, 1, 1);
    config.dynamicSmemBytes = smem_bytes<true>();
    cudaLaunchAttribute attribute;
    attribute.id = cudaLaunchAttributeClusterDimension;
    attribute.val.clusterDim.x = 2;
    attribute.val.clusterDim.y = 1;
    attribute.val.clusterDim.z = 1;
    config.attrs = &attribute;
    config.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, w8a8_gemm_sm100_kernel<true, true>, &config) != cudaSuccess ||
        clusters <= 0) {
        (void)cudaGetLastError();
        return sm_count / 2;
    }
    cached[device].store(clusters, std::memory_order_relaxed);
    return clusters;
}

template <bool FANOUT, bool PAIR>
cudaError_t launch_kernel(uint32_t tiles, int sm_count, const CUtensorMap *map_a, const CUtensorMap *map_w,
                          const CUtensorMap *map_out, const GemmParams &params, cudaStream_t stream) {
    cudaLaunchAttribute attributes[2] = {};
    attributes[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attributes[0].val.programmaticStreamSerializationAllowed = 1;
    if constexpr (!PAIR) {
        const uint32_t grid = tiles < static_cast<uint32_t>(sm_count) ? tiles : static_cast<uint32_t>(sm_count);
        cudaLaunchConfig_t config = {};
        config.gridDim = dim3(grid, 1, 1);
        config.blockDim = dim3(NUM_THREADS, 1, 1);
        config.dynamicSmemBytes = smem_bytes<false>();
        config.stream = stream;
        config.attrs = attributes;
        config.numAttrs = 1;
        return cudaLaunchKernelEx(&config, w8a8_gemm_sm100_kernel<FANOUT, false>, *map_a, *map_w, *map_out, params);
    } else {
        const uint32_t pairs = static_cast<uint32_t>(resident_pairs(sm_count));
        const uint32_t clusters = tiles < pairs ? tiles : pairs;
        cudaLaunchConfig_t config = {};
        config.gridDim = dim3(2 * clusters, 1, 1);
        config.blockDim = dim3(NUM_THREADS, 1, 1);
        config.dynamicSmemBytes = smem_bytes<true>();
        config.stream = stream;
        attributes[1].id = cudaLaunchAttributeClusterDimension;
        attributes[1].val.clusterDim.x = 2;
        attributes[1].val.clusterDim.y = 1;
        attributes[1].val.clusterDim.z = 1;
        config.attrs = attributes;
        config.numAttrs = 2;
        return cudaLaunchKernelEx(&config, w8a8_gemm_sm100_kernel<FANOUT, true>, *map_a, *map_w, *map_out, params);
    }
}

}  // namespace

// Single-CTA tiles (128 x 256) for one row block; CTA pairs (256 x 256 per pair, a third less A
// and B traffic per output than the single-CTA tile, 256-byte K stages) from two row blocks on.
// Measured on B200 (M = 4096, L2 flushed): the 70B FFN gate GEMM takes 746 us single-CTA and
// 666 us in pairs, down 692 and 602 us; with peer destinations (fused all-gather, 2 GPUs) the
// step measured 4137 TOPS in pairs against 4071-4077 single-CTA in the same call.
cudaError_t launch_w8a8_gemm_sm100(const CUtensorMap *map_a, const CUtensorMap *map_w, uint32_t m, uint32_t n,
                                   uint32_t k, const GemmEpilogue &epilogue, unsigned int *error_word, int sm_count,
                                   cudaStream_t stream) {
    const bool pair = m > kGemmBlockM;
    return launch_w8a8_gemm_sm100_mode(map_a, map_w, m, n, k, epilogue, error_word, sm_count, pair, stream);
}

namespace {
// Shared-memory attribute of every variant, once per device (setting it also loads the kernel
// under CUDA's lazy module loading).
cudaError_t configure_all_variants() {
    static PerDeviceOnce configured;
    return configured.run([] {
        cudaError_t error = configure_kernel<false, false>();
        if (error == cudaSuccess) error = configure_kernel<true, false>();
        if (error == cudaSuccess) error = configure_kernel<false, true>();
        if (error == cudaSuccess) error = configure_kernel<true, true>();
        return error;
    });
}
}  // namespace

cudaError_t preload_w8a8_gemm_sm100(int sm_count) {
    const cudaError_t error = configure_all_variants();
    if (error != cudaSuccess) return error;
    (void)resident_pairs(sm_count);  // the cluster occupancy query, cached per device
    return cudaSuccess;
}

cudaError_t launch_w8a8_gemm_sm100_mode(const CUtensorMap *map_a, const CUtensorMap *map_w, uint32_t m, uint32_t n,
                                        uint32_t k, const GemmEpilogue &epilogue, unsigned int *error_word,
                                        int sm_count, bool pair, cudaStream_t stream) {
    if (m == 0 || n == 0) return cudaSuccess;
    if (k == 0) return cudaErrorInvalidValue;
    const cudaError_t configure_error = configure_all_variants();
    if (configure_error != cudaSuccess) return configure_error;
    pair = pair && sm_count >= 2;
    GemmParams params;
    params.m = m;
    params.n = n;
    params.k = k;
    params.num_kb = pair ? (k + Pipe<true>::K_STAGE - 1) / Pipe<true>::K_STAGE : (k + BK - 1) / BK;
    params.m_blocks = (m + (pair ? 2 * BM : BM) - 1) / (pair ? 2 * BM : BM);
    params.n_blocks = (n + BN - 1) / BN;
    params.mode = static_cast<int>(epilogue.mode);
    params.row_scales = epilogue.row_scales;
    params.col_scales = epilogue.col_scales;
    params.bias = epilogue.bias;
    params.out = epilogue.out;
    params.out_stride = epilogue.out_stride;
    if (epilogue.peer_count > kGemmMaxPeers) return cudaErrorInvalidValue;
    params.peer_count = epilogue.peer_count;
    for (uint32_t d = 0; d < kGemmMaxPeers; ++d) params.peer_out[d] = d < epilogue.peer_count ? epilogue.peer_out[d] : nullptr;
    if (epilogue.rows_per_batch == 0 || epilogue.col_stride == 0) return cudaErrorInvalidValue;
    params.rows_per_batch = epilogue.rows_per_batch;
    params.batch_stride = epilogue.batch_stride;
    params.col_stride = epilogue.col_stride;
    params.error_word = error_word;
    params.splits = 1;
    {
        const uint64_t block_bytes = static_cast<uint64_t>(pair ? 2 * BM : BM) * k;
        uint64_t group = block_bytes != 0 ? kTileGroupBytes / block_bytes : kTileGroupRows;
        if (group < kTileGroupRows) group = kTileGroupRows;
        if (group > params.m_blocks) group = params.m_blocks;
        params.group_rows = group != 0 ? static_cast<uint32_t>(group) : 1u;
    }
    params.kb_per_split = params.num_kb;
    params.split_rows = 0;
    const uint32_t tiles = params.m_blocks * params.n_blocks;
    const bool fanout = params.peer_count != 0;
    // A local row-major output leaves through TMA stores (full 128-byte lines; per-lane 16-byte
    // stores of 32 different rows moved 3x the output bytes through L1 and cost 20% at K = 8192).
    CUtensorMap map_out;
    std::memset(&map_out, 0, sizeof(map_out));
    params.tma_store = !fanout && params.col_stride == 1 && params.rows_per_batch == 0xFFFFFFFFu &&
                       params.out_stride >= n &&
                       encode_tensor_map_2d_b32(&map_out, params.out, n, m, params.out_stride * 4u, 32u, 32u);
    if (pair) {
        return fanout ? launch_kernel<true, true>(tiles, sm_count, map_a, map_w, &map_out, params, stream)
                      : launch_kernel<false, true>(tiles, sm_count, map_a, map_w, &map_out, params, stream);
    }
    return fanout ? launch_kernel<true, false>(tiles, sm_count, map_a, map_w, &map_out, params, stream)
                  : launch_kernel<false, false>(tiles, sm_count, map_a, map_w, &map_out, params, stream);
}

cudaError_t launch_w8a8_gemm_sm100_splitk(const CUtensorMap *map_a, const CUtensorMap *map_w, uint32_t m, uint32_t n,
                                          uint32_t k, int32_t *workspace, uint32_t splits, unsigned int *error_word,
                                          int sm_count, cudaStream_t stream, uint32_t *used_splits) {
    if (m == 0 || n == 0 || k == 0 || splits < 2 || n % 4 != 0 || (reinterpret_cast<uintptr_t>(workspace) & 15u) != 0) {
        return cudaErrorInvalidValue;
    }
    const cudaError_t configure_error = configure_all_variants();
    if (configure_error != cudaSuccess) return configure_error;
    GemmParams params{};
    params.m = m;
    params.n = n;
    params.k = k;
    params.num_kb = (k + BK - 1) / BK;
    params.m_blocks = (m + BM - 1) / BM;
    params.n_blocks = (n + BN - 1) / BN;
    params.mode = static_cast<int>(EpilogueMode::kStoreS32);
    params.out = workspace;
    params.out_stride = n;
    params.peer_count = 0;
    params.rows_per_batch = 0xFFFFFFFFu;
    params.batch_stride = 0;
    params.col_stride = 1;
    params.error_word = error_word;
    // every slice gets at least one K stage
    params.kb_per_split = (params.num_kb + splits - 1) / splits;
    params.splits = (params.num_kb + params.kb_per_split - 1) / params.kb_per_split;
    params.split_rows = params.m_blocks * BM;
    params.group_rows = kTileGroupRows;
    CUtensorMap map_out;
    std::memset(&map_out, 0, sizeof(map_out));
    params.tma_store = encode_tensor_map_2d_b32(&map_out, workspace, n,
                                                static_cast<uint64_t>(params.splits) * params.split_rows,
                                                static_cast<uint64_t>(n) * 4u, 32u, 32u);
    if (!params.tma_store || params.splits < 2) return cudaErrorInvalidValue;
    *used_splits = params.splits;
    return launch_kernel<false, false>(params.m_blocks * params.n_blocks * params.splits, sm_count, map_a, map_w, &map_out,
                                       params, stream);
}

cudaError_t run_w8a8_gemm(const int8_t *a, size_t a_stride, const int8_t *w, size_t w_stride, uint32_t m, uint32_t n,
                          uint32_t k, const GemmEpilogue &epilogue, unsigned int *error_word, int sm_count,
                          cudaStream_t stream) {
    CUtensorMap map_a, map_w;
    if (!encode_tensor_map_2d_u8(&map_a, a, k, m, a_stride, BK, BM) ||
        !encode_tensor_map_2d_u8(&map_w, w, k, n, w_stride, BK, W_BOX_ROWS)) {
        return cudaErrorInvalidValue;
    }
    return launch_w8a8_gemm_sm100(&map_a, &map_w, m, n, k, epilogue, error_word, sm_count, stream);
}

}  // namespace qpucuda
