// The cross key/value projection of a sequence start on the tcgen05 tensor
// cores (sm_100a): recordSequenceStart, Lib/WhisperEACP/Decoder/Decoder.cpp:
// 121-146, for every window of a batch in one persistent launch.  The
// product and the cache layout are described in cross_kv.cuh.
//
// A tile is 128 encoder rows (the MMA's M) by 256 weight rows (its N) over
// the whole width, in 64-column k-blocks.  Each CTA walks tiles c, c + grid,
// ... (window-major, then weight tile, then row tile, so the CTAs at work at
// one time share a weight tile through L2).  Warp roles:
//
//   warps 6..13  read the tile's fp32 encoder rows, a k-block at a time, and
//                write them into shared memory as two 16-bit tiles, hi and
//                lo = x - hi, in the 128-byte-swizzled K-major layout: the
//                fp32 -> 16-bit narrowing happens here, and hi + lo carries
//                about twice the 16-bit precision into the product;
//   warp 5       lane 0 copies the weight tile's k-block (32 KB, laid out for
//                the tensor cores at upload) with one cp.async.bulk;
//   warp 4       lane 0 issues tcgen05.mma (M 128, N 256, K 16): A_hi . B and
//                A_lo . B into the same fp32 accumulator in tensor memory;
//                two accumulators of 256 columns alternate between tiles so
//                the epilogue of one overlaps the products of the next;
//   warps 0..3   read the accumulator back (tcgen05.ld, a TMEM lane = an
//                encoder row), narrow to the cache's 16-bit type and store
//                each row's pieces straight into the (layer, window, head)
//                block they belong to, rotated for the attention's reads.
//
// Three stages of (A hi, A lo, B) = 64 KB ring between producers and the
// MMA.  Every wait is bounded (2 s): one that gives up records which, raises
// the CTA's abort flag so every other role gives up too, and the kernel
// drains its copies and products, frees its tensor memory and returns.
#include "common.cuh"
#include "cross_kv.cuh"
#include "umma.cuh"

#include <stdexcept>
#include <string>

namespace wsp {
namespace {

constexpr int kStages = 3;
constexpr int kEpilogueWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kCopyWarp = 5;
constexpr int kFirstRowWarp = 6;
constexpr int kRowWarps = 8;
constexpr int kCkvThreads = 32 * (kFirstRowWarp + kRowWarps);
constexpr int kTileM = 128;
constexpr int kAStageBytes = kTileM * 128;               // 128 rows x 64 16-bit columns
constexpr int kBStageBytes = kCrossTileRows * 128;        // 256 rows x 64 16-bit columns
constexpr int kStageBytes = 2 * kAStageBytes + kBStageBytes;
constexpr uint32_t kTmemColumns = 512;                    // two accumulators of 256 columns
constexpr int kAccColumns = 256;
constexpr unsigned long long kTimeoutNs = 2000000000ull;

// Which wait gave up (the status word).
enum CrossKvWait : int { kWaitRows = 1, kWaitWeights = 2, kWaitFree = 3, kWaitAccumulator = 4, kWaitDrained = 5,
                         kWaitReadBack = 6 };

__device__ __forceinline__ unsigned long long clock_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool phase_done(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}\n"
        : "=r"(done)
        : "r"(smem_address(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the phase of `parity`; false once the CTA's abort flag is up or
// after kTimeoutNs (then it records `kind` and raises the flag).
__device__ bool wait_phase(uint64_t* bar, uint32_t parity, volatile int* abort, int* status, int kind) {
    if (phase_done(bar, parity)) return true;
    const unsigned long long start = clock_ns();
    for (unsigned spin = 1;; ++spin) {
        if (phase_done(bar, parity)) return true;
        if ((spin & 15) != 0) continue;
        if (*abort) return false;
        if (clock_ns() - start > kTimeoutNs) {
            atomicCAS(status, 0, kind);
            *abort = 1;
            return false;
        }
    }
}

__device__ __forceinline__ void arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_address(bar)) : "memory");
}

struct TileCoords {
    int window, weight_tile, row_tile;
};
__device__ __forceinline__ TileCoords tile_coords(long long tile, int row_tiles, int weight_tiles) {
    TileCoords t;
    t.row_tile = (int)(tile % row_tiles);
    const long long rest = tile / row_tiles;
    t.weight_tile = (int)(rest % weight_tiles);
    t.window = (int)(rest / weight_tiles);
    return t;
}

// Warps kFirstRowWarp..: rows 16 w .. 16 w + 15 of each tile, a k-block at a
// time.  Lane l reads float4 l % 16 of row 2 i + l / 16, so a warp's load
// covers two rows' 256 contiguous bytes.
template <typename WT>
__device__ void load_rows(const CrossKvArgs& a, unsigned char* smem, uint64_t* full, uint64_t* empty, int row_tiles,
                          int weight_tiles, long long tiles, volatile int* abort) {
    const int w = (threadIdx.x >> 5) - kFirstRowWarp, lane = threadIdx.x & 31;
    const int pair = lane >> 4, c4 = lane & 15;
    unsigned long long q = 0;
    for (long long tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const TileCoords t = tile_coords(tile, row_tiles, weight_tiles);
        const float* window = a.encoder + (size_t)t.window * a.row_stride * a.width;
        for (int kb = 0; kb < a.kblocks; ++kb, ++q) {
            const int stage = (int)(q % kStages);
            if (q >= (unsigned long long)kStages &&
                !wait_phase(empty + stage, (uint32_t)((q / kStages - 1) & 1), abort, a.status, kWaitFree))
                return;
            const int k = kb * 64 + c4 * 4;
            float4 v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int row = t.row_tile * kTileM + 16 * w + 2 * i + pair;
                v[i] = row < a.rows && k < a.width
                           ? __ldg(reinterpret_cast<const float4*>(window + (size_t)row * a.width + k))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            unsigned char* hi_tile = smem + (size_t)stage * kStageBytes;
            unsigned char* lo_tile = hi_tile + kAStageBytes;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = 16 * w + 2 * i + pair;
                const uint32_t offset = (uint32_t)(r * 128 + ((((c4 >> 1) ^ (r & 7))) << 4) + ((c4 & 1) << 3));
                uint32_t h0, l0, h1, l1;
                split_pair<WT>(v[i].x, v[i].y, h0, l0);
                split_pair<WT>(v[i].z, v[i].w, h1, l1);
                asm volatile("st.shared.v2.u32 [%0], {%1, %2};\n" ::"r"(smem_address(hi_tile + offset)), "r"(h0),
                             "r"(h1)
                             : "memory");
                asm volatile("st.shared.v2.u32 [%0], {%1, %2};\n" ::"r"(smem_address(lo_tile + offset)), "r"(l0),
                             "r"(l1)
                             : "memory");
            }
            // The tensor cores read these through the async proxy.
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            __syncwarp();
            if (lane == 0) arrive(full + stage);
        }
    }
}

// Warp kCopyWarp, lane 0: the weight tile's k-blocks, one bulk copy each;
// then waits for the copies still landing.
__device__ void load_weights(const CrossKvArgs& a, unsigned char* smem, uint64_t* landed, uint64_t* empty,
                             int row_tiles, int weight_tiles, long long tiles, volatile int* abort) {
    const unsigned char* weights = static_cast<const unsigned char*>(a.weight);
    unsigned long long q = 0;
    for (long long tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
        const TileCoords t = tile_coords(tile, row_tiles, weight_tiles);
        bool go = true;
        for (int kb = 0; kb < a.kblocks; ++kb, ++q) {
            const int stage = (int)(q % kStages);
            if (q >= (unsigned long long)kStages &&
                !wait_phase(empty + stage, (uint32_t)((q / kStages - 1) & 1), abort, a.status, kWaitFree)) {
                go = false;
                break;
            }
            const uint32_t bar = smem_address(landed + stage);
            const uint32_t dst = smem_address(smem + (size_t)stage * kStageBytes + 2 * kAStageBytes);
            const unsigned char* src = weights + ((size_t)t.weight_tile * a.kblocks + kb) * kBStageBytes;
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(kBStageBytes)
                         : "memory");
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
                "l"(src), "r"(kBStageBytes), "r"(bar)
                : "memory");
        }
        if (!go) break;
    }
    // No copy may outlive the CTA: wait (bounded, even after an abort) for
    // the last stages' copies to land.
    for (unsigned long long v = q > (unsigned long long)kStages ? q - kStages : 0; v < q; ++v) {
        uint64_t* bar = landed + v % kStages;
        const uint32_t parity = (uint32_t)((v / kStages) & 1);
        const unsigned long long start = clock_ns();
        while (!phase_done(bar, parity))
            if (clock_ns() - start > kTimeoutNs) {
                atomicCAS(a.status, 0, kWaitDrained);
                *abort = 1;
                break;
            }
    }
}

// Warp kMmaWarp, lane 0: the products of every tile into alternating
// accumulators; then one commit whose completion means every product issued
// has finished (so the tensor memory can be freed).
template <typename WT>
__device__ void issue_products(const CrossKvArgs& a, unsigned char* smem, uint64_t* full, uint64_t* landed,
                               uint64_t* empty, uint64_t* acc_full, uint64_t* acc_empty, uint64_t* drained,
                               uint32_t tmem, long long tiles, volatile int* abort) {
    const uint32_t idesc = umma_idesc<WT>(kCrossTileRows);
    unsigned long long q = 0;
    long long it = 0;
    for (long long tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++it) {
        const int acc = (int)(it & 1);
        if (it >= 2 && !wait_phase(acc_empty + acc, (uint32_t)((it / 2 - 1) & 1), abort, a.status, kWaitAccumulator))
            break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + (uint32_t)(acc * kAccColumns);
        bool go = true;
        for (int kb = 0; kb < a.kblocks; ++kb, ++q) {
            const int stage = (int)(q % kStages);
            const uint32_t parity = (uint32_t)((q / kStages) & 1);
            if (!wait_phase(full + stage, parity, abort, a.status, kWaitRows) ||
                !wait_phase(landed + stage, parity, abort, a.status, kWaitWeights)) {
                go = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t base = smem_address(smem + (size_t)stage * kStageBytes);
            const uint32_t b = base + 2 * kAStageBytes;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                umma_mma(d, umma_desc(base + 32 * kk), umma_desc(b + 32 * kk), idesc, (kb | kk) != 0);
                umma_mma(d, umma_desc(base + kAStageBytes + 32 * kk), umma_desc(b + 32 * kk), idesc, 1u);
            }
            umma_commit(empty + stage);  // the stage is free once these have read it
        }
        if (!go) break;
        umma_commit(acc_full + acc);
    }
    umma_commit(drained);
    const unsigned long long start = clock_ns();
    while (!phase_done(drained, 0))
        if (clock_ns() - start > kTimeoutNs) {
            atomicCAS(a.status, 0, kWaitDrained);
            *abort = 1;
            break;
        }
}

// The cache block of (window, group = layer * H + head): [layer][window][head].
__device__ __forceinline__ size_t cache_block(const CrossKvArgs& a, int window, int group) {
    const int layer = group / a.heads, head = group % a.heads;
    return ((size_t)layer * a.windows + window) * a.heads + head;
}

// Warps 0..3: row 32 w + lane of each tile from its accumulator into the
// cache.  With 64-wide heads a 256-column accumulator is two (layer, head)
// groups of K | V; each 32-column read is four 16-byte pieces of one row,
// stored at their rotated places (cross_piece) in their (layer, window,
// head) block.
template <typename WT>
__device__ void store_tiles(const CrossKvArgs& a, uint64_t* acc_full, uint64_t* acc_empty, uint32_t tmem,
                            int row_tiles, int weight_tiles, long long tiles, volatile int* abort) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int two_d = 2 * a.head_width;
    WT* out = static_cast<WT*>(a.out);
    long long it = 0;
    for (long long tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++it) {
        const int acc = (int)(it & 1);
        if (!wait_phase(acc_full + acc, (uint32_t)((it / 2) & 1), abort, a.status, kWaitReadBack)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const TileCoords t = tile_coords(tile, row_tiles, weight_tiles);
        const int row = t.row_tile * kTileM + 32 * warp + lane;
        const bool row_ok = row < a.rows;
        for (int c0 = 0; c0 < kAccColumns; c0 += 32) {
            uint32_t v[32];
            tmem_load32(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(acc * kAccColumns + c0), v);
            const int n0 = t.weight_tile * kCrossTileRows + c0;
            if (!row_ok || n0 >= a.columns) continue;
            if (a.linear_out) {
                // Row `row`'s 32 columns n0..: bias, GELU, residual, as
                // float4s (columns is a multiple of 4).
                float* out_row = a.linear_out + (size_t)row * a.columns;
                const float* res_row = a.residual ? a.residual + (size_t)row * a.columns : nullptr;
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    const int n = n0 + j;
                    if (n >= a.columns) break;
                    float x[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        x[e] = __uint_as_float(v[j + e]) + (a.bias ? __ldg(a.bias + n + e) : 0.f);
                        if (a.gelu) x[e] = gelu_exact(x[e]);
                    }
                    if (res_row) {
                        const float4 r = *reinterpret_cast<const float4*>(res_row + n);
                        x[0] += r.x;
                        x[1] += r.y;
                        x[2] += r.z;
                        x[3] += r.w;
                    }
                    *reinterpret_cast<float4*>(out_row + n) = make_float4(x[0], x[1], x[2], x[3]);
                }
                continue;
            }
            if (a.head_width == 64) {
                const int group = n0 / 128, piece0 = (n0 % 128) / 8;
                WT* block = out + (cache_block(a, t.window, group) * a.row_stride + row) * 128;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint4 piece;
                    piece.x = Half16<WT>::pack2(__uint_as_float(v[8 * j]), __uint_as_float(v[8 * j + 1]));
                    piece.y = Half16<WT>::pack2(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3]));
                    piece.z = Half16<WT>::pack2(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5]));
                    piece.w = Half16<WT>::pack2(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7]));
                    *reinterpret_cast<uint4*>(block + cross_piece(piece0 + j, row) * 8) = piece;
                }
            } else {
                for (int j = 0; j < 32; ++j) {
                    const int n = n0 + j;
                    if (n >= a.columns) break;
                    const int group = n / two_d, c = n % two_d;
                    out[(cache_block(a, t.window, group) * a.row_stride + row) * two_d + c] =
                        Half16<WT>::from_float(__uint_as_float(v[j]));
                }
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) arrive(acc_empty + acc);
    }
}

template <typename WT>
__global__ void __launch_bounds__(kCkvThreads, 1) cross_kv_kernel(CrossKvArgs a) {
    extern __shared__ unsigned char dynamic_smem[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(dynamic_smem) + 1023) & ~static_cast<uintptr_t>(1023));
    __shared__ __align__(8) uint64_t full[kStages], landed[kStages], empty[kStages];
    __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], drained;
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    const int warp = threadIdx.x >> 5;
    const int row_tiles = (a.rows + kTileM - 1) / kTileM;
    const int weight_tiles = (a.columns + kCrossTileRows - 1) / kCrossTileRows;
    const long long tiles = (long long)a.windows * weight_tiles * row_tiles;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int i = 0; i < kStages; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_address(full + i)), "r"(kRowWarps)
                         : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_address(landed + i)) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_address(empty + i)) : "memory");
        }
        for (int i = 0; i < 2; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_address(acc_full + i)) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_address(acc_empty + i)),
                         "r"(kEpilogueWarps)
                         : "memory");
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_address(&drained)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_address(&tmem_slot)),
                     "r"(kTmemColumns));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_slot;
    volatile int* abort = &abort_flag;

    if (warp >= kFirstRowWarp) {
        load_rows<WT>(a, smem, full, empty, row_tiles, weight_tiles, tiles, abort);
    } else if (warp == kCopyWarp) {
        if ((threadIdx.x & 31) == 0) load_weights(a, smem, landed, empty, row_tiles, weight_tiles, tiles, abort);
    } else if (warp == kMmaWarp) {
        if ((threadIdx.x & 31) == 0)
            issue_products<WT>(a, smem, full, landed, empty, acc_full, acc_empty, &drained, tmem, tiles, abort);
    } else {
        store_tiles<WT>(a, acc_full, acc_empty, tmem, row_tiles, weight_tiles, tiles, abort);
    }

    // Every product has completed (the issuer waited for its last commit):
    // the tensor memory can go.
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemColumns));
}

template <typename WT>
void launch_typed(const CrossKvArgs& a, int sm_count, cudaStream_t stream) {
    const size_t smem = cross_kv_shared_bytes();
    cudaError_t e = cudaFuncSetAttribute(cross_kv_kernel<WT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) throw std::runtime_error(std::string("cross key/value kernel: ") + cudaGetErrorString(e));
    const int row_tiles = (a.rows + kTileM - 1) / kTileM;
    const int weight_tiles = (a.columns + kCrossTileRows - 1) / kCrossTileRows;
    const long long tiles = (long long)a.windows * weight_tiles * row_tiles;
    const int grid = (int)std::min<long long>(tiles, sm_count);
    cross_kv_kernel<WT><<<grid, kCkvThreads, smem, stream>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string("cross key/value launch: ") + cudaGetErrorString(e));
}

}  // namespace

size_t cross_kv_shared_bytes() { return 1024 + (size_t)kStages * kStageBytes; }

void launch_cross_kv(bool half, const CrossKvArgs& a, int sm_count, cudaStream_t stream) {
    if (a.linear_out) {
        if (a.windows != 1 || a.rows <= 0 || a.rows > a.row_stride || a.width <= 0 || a.width % 4 != 0 ||
            a.kblocks != (a.width + 63) / 64 || a.columns <= 0 || a.columns % 4 != 0 ||
            (reinterpret_cast<uintptr_t>(a.encoder) & 15) != 0 || (reinterpret_cast<uintptr_t>(a.weight) & 15) != 0 ||
            (reinterpret_cast<uintptr_t>(a.linear_out) & 15) != 0 ||
            (reinterpret_cast<uintptr_t>(a.residual) & 15) != 0)
            throw std::runtime_error("tensor-core product: arguments out of range");
        if (half) launch_typed<__half>(a, sm_count, stream);
        else launch_typed<__nv_bfloat16>(a, sm_count, stream);
        return;
    }
    if (a.windows <= 0 || a.rows <= 0 || a.rows > a.row_stride || a.width <= 0 || a.width % 4 != 0 ||
        a.kblocks != (a.width + 63) / 64 || a.columns <= 0 || a.head_width <= 0 || a.groups <= 0 ||
        a.heads <= 0 || a.groups % a.heads != 0 ||
        a.columns != a.groups * 2 * a.head_width || (reinterpret_cast<uintptr_t>(a.encoder) & 15) != 0 ||
        (reinterpret_cast<uintptr_t>(a.weight) & 15) != 0 || (reinterpret_cast<uintptr_t>(a.out) & 15) != 0)
        throw std::runtime_error("cross key/value projection: arguments out of range");
    if (half) launch_typed<__half>(a, sm_count, stream);
    else launch_typed<__nv_bfloat16>(a, sm_count, stream);
}

}  // namespace wsp
