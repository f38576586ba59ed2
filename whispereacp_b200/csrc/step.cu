// The persistent decode kernel: the step's op list, once per step, with a
// grid-wide barrier after each op.  See step.cuh for the op list.
//
// Reference semantics (paths within eyalamirmusic/WhisperEACP):
//   embed            Lib/WhisperEACP/Kernels/Embed.h:38-64
//   layer norm       Lib/WhisperEACP/Kernels/LayerNorm.h:19-98 (two-pass, eps 1e-5)
//   products         Lib/WhisperEACP/Kernels/Linear.h:128-276 (bias, exact GELU, residual)
//   attention        Lib/WhisperEACP/Kernels/SingleQueryAttention.h:62-373,397-501,
//                    Attention.h:75-209 (scale on the scores; causal for a prompt)
//   masked argmax    Lib/WhisperEACP/Kernels/Argmax.h:83-201 (first maximum; none -> 0)
//
// Data written by one CTA and read by another inside the launch is read with
// ld.global.cg (L2, never a stale L1 line); the grid barrier orders it.
#include "step.cuh"
#include "step_launch.h"

#include <algorithm>
#include <stdexcept>
#include <string>

namespace wsp {
namespace {

// ------------------------------------------------------------ memory access

__device__ __forceinline__ uint4 ld_cg4(const void* p) {
    uint4 v;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ float ld_cg(const float* p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];\n" : "=f"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ld_cg(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.global.cg.u32 %0, [%1];\n" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ unsigned short ld_cg_u16(const void* p) {
    unsigned short v;
    asm volatile("ld.global.cg.u16 %0, [%1];\n" : "=h"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ unsigned short ld_nc_u16(const void* p) {
    unsigned short v;
    asm volatile("ld.global.nc.u16 %0, [%1];\n" : "=h"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

template <typename WT>
__device__ __forceinline__ float bits_to_float(unsigned short b) {
    return Half16<WT>::to_float(*reinterpret_cast<const WT*>(&b));
}

// -------------------------------------------------------------- grid barrier

constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;  // 2 s

// A monotonic arrival counter: each CTA adds one with release semantics and
// waits, with acquire loads, until every CTA has arrived `epoch` times.  The
// wait gives up after kWaitTimeoutNs (or as soon as another CTA gave up): it
// records kErrBarrierTimeout, raises the abort word and the kernel returns.
__device__ bool grid_barrier(unsigned* count, unsigned& epoch, int* state) {
    __shared__ int aborted;
    __syncthreads();
    ++epoch;
    if (threadIdx.x == 0) {
        asm volatile("red.release.gpu.global.add.u32 [%0], %1;\n" ::"l"(count), "r"(1u) : "memory");
        const unsigned target = epoch * gridDim.x;
        const unsigned long long start = global_ns();
        while (ld_acquire(count) < target) {
            if (ld_volatile(state + kAbort)) break;
            if (global_ns() - start > kWaitTimeoutNs) {
                atomicOr(state + kError, kErrBarrierTimeout);
                atomicExch(state + kAbort, 1);
                break;
            }
        }
        aborted = ld_volatile(state + kAbort);
    }
    __syncthreads();
    return aborted == 0;
}

// ------------------------------------------------------------ weight stream

// Weight tiles stream through a ring of shared-memory stages, each filled by
// one cp.async.bulk copy that completes an mbarrier.  The CTA's sequence of
// weight units -- (op, tile, k-block) over the products and the logits of
// every step, in the order the ops consume them -- is fixed, so thread 0
// issues ahead as far as the ring allows: the next op's first tiles are in
// flight while this op (an attention, say) and the grid barrier run.
constexpr int kUnitChunks = 32;                  // 1024 k of a 16-row tile
constexpr int kUnitBytes = kUnitChunks * 1024;   // 32 KB

__device__ __forceinline__ uint32_t smem_address(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

struct Cursor {
    int step, op, item, block;
};

struct Stream {
    unsigned char* ring;        // stages x kUnitBytes
    uint64_t* full;             // one mbarrier per stage
    int stages;
    unsigned long long consumed;  // units every thread has finished with
    unsigned long long issued;    // thread 0 only
    Cursor cursor;                // thread 0 only: the next unit to issue
};

// The weight, extent and inner size a product-like op streams.
__device__ __forceinline__ bool op_streams(const StepParams& p, const StepOp& op, const void** weight, int* n,
                                           int* kp, int* rows) {
    if (op.kind == kOpProduct) {
        *weight = op.weight; *n = op.n; *kp = op.kp; *rows = p.rows;
        return true;
    }
    if (op.kind == kOpLogits) {
        *weight = p.token_table; *n = p.vocabulary; *kp = p.kpd; *rows = p.out_rows;
        return true;
    }
    return false;
}

// Thread 0: the next unit of this CTA's sequence, or false past the last step.
template <int RT>
__device__ bool next_unit(const StepParams& p, Cursor& c, const unsigned char** src, unsigned* bytes) {
    while (c.step < p.steps) {
        if (c.op >= p.n_ops) {
            c.op = 0;
            c.item = blockIdx.x;
            c.block = 0;
            ++c.step;
            continue;
        }
        const void* weight;
        int n, kp, rows;
        if (op_streams(p, p.ops[c.op], &weight, &n, &kp, &rows)) {
            const int n_tiles = (n + 15) / 16;
            const int items = n_tiles * ((rows + RT - 1) / RT);
            if (c.item < items) {
                const int chunks = kp / 32;
                const int blocks = (chunks + kUnitChunks - 1) / kUnitChunks;
                const int n_tile = c.item % n_tiles;
                const int chunk0 = c.block * kUnitChunks;
                *src = static_cast<const unsigned char*>(weight) + ((size_t)n_tile * chunks + chunk0) * 1024;
                *bytes = (unsigned)min(kUnitChunks, chunks - chunk0) * 1024u;
                if (++c.block == blocks) {
                    c.block = 0;
                    c.item += gridDim.x;
                }
                return true;
            }
        }
        ++c.op;
        c.item = blockIdx.x;
        c.block = 0;
    }
    return false;
}

// Thread 0: fills every free stage.
template <int RT>
__device__ void issue_ahead(const StepParams& p, Stream& s) {
    while (s.issued < s.consumed + (unsigned long long)s.stages) {
        const unsigned char* src;
        unsigned bytes;
        if (!next_unit<RT>(p, s.cursor, &src, &bytes)) return;
        const int stage = (int)(s.issued % s.stages);
        const uint32_t bar = smem_address(s.full + stage);
        const uint32_t dst = smem_address(s.ring + (size_t)stage * kUnitBytes);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
                     "l"(src), "r"(bytes), "r"(bar)
                     : "memory");
        ++s.issued;
    }
}

// Waits (bounded) for unit `index` to land; false if the wait gave up.
__device__ bool wait_unit(const StepParams& p, const Stream& s, unsigned long long index) {
    const uint32_t bar = smem_address(s.full + (int)(index % s.stages));
    const uint32_t parity = (uint32_t)((index / s.stages) & 1);
    const unsigned long long start = global_ns();
    while (true) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred P;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, P;\n\t}\n"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
        if (global_ns() - start > kWaitTimeoutNs) {
            atomicOr(p.state + kError, kErrBarrierTimeout);
            atomicExch(p.state + kAbort, 1);
            return false;
        }
    }
}

// After a unit: every thread is done reading its stage, which thread 0 may
// now refill.
template <int RT>
__device__ __forceinline__ void release_unit(const StepParams& p, Stream& s) {
    __syncthreads();
    ++s.consumed;
    if (threadIdx.x == 0) issue_ahead<RT>(p, s);
}

// -------------------------------------------------------------------- embed

template <typename WT>
__device__ void op_embed(const StepParams& p, int position) {
    const WT* table = static_cast<const WT*>(p.token_table);
    for (int r = blockIdx.x; r < p.rows; r += gridDim.x) {
        const int b = r / p.tokens, t = r % p.tokens;
        const int at = position + t;
        uint32_t token = ld_cg(p.ring + (size_t)b * p.ring_stride + at);
        if (token >= (uint32_t)p.vocabulary) {
            if (threadIdx.x == 0) atomicOr(p.state + kError, kErrToken);
            token = 0;
        }
        const float* pos = p.position_table + (size_t)at * p.width;
        float* out = p.h + (size_t)r * p.width;
        const int chunks = p.kpd / 32;
        for (int c = threadIdx.x; c < p.width; c += kThreads)
            out[c] = Half16<WT>::to_float(table[packed_offset((int)token, c, chunks)]) + pos[c];
    }
}

// ------------------------------------------------------- layer-norm prologue

constexpr int kNormMaxPerLane = 48;  // widths up to 1536

// LayerNorm of rows_in_tile rows of h into the 16-bit tile xs [rows][ldx]:
// output row rl reads h row (r0 + rl)*row_step + row_offset.  One warp a row,
// the row in registers: the mean, then the centred variance, as
// LayerNorm.h:19-98 does.  hidden_out, when given, receives the fp32 rows.
template <typename WT>
__device__ void layer_norm_tile(const StepParams& p, const float* gamma, const float* beta, int r0,
                                int rows_in_tile, int row_step, int row_offset, WT* xs, int ldx,
                                float* hidden_out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = p.width;
    for (int rl = warp; rl < rows_in_tile; rl += kWarps) {
        const float* x = p.h + ((size_t)(r0 + rl) * row_step + row_offset) * d;
        float v[kNormMaxPerLane];
        float total = 0.f;
#pragma unroll
        for (int i = 0; i < kNormMaxPerLane; ++i) {
            const int c = lane + 32 * i;
            v[i] = c < d ? ld_cg(x + c) : 0.f;
            total += v[i];
        }
        const float mean = warp_sum(total) / (float)d;
        float centred = 0.f;
#pragma unroll
        for (int i = 0; i < kNormMaxPerLane; ++i) {
            const int c = lane + 32 * i;
            const float dv = c < d ? v[i] - mean : 0.f;
            centred += dv * dv;
        }
        const float scale = rsqrtf(warp_sum(centred) / (float)d + 1e-5f);
        WT* out = xs + (size_t)rl * ldx;
#pragma unroll
        for (int i = 0; i < kNormMaxPerLane; ++i) {
            const int c = lane + 32 * i;
            if (c < d) {
                const float y = (v[i] - mean) * scale * gamma[c] + beta[c];
                out[c] = Half16<WT>::from_float(y);
                if (hidden_out) hidden_out[(size_t)(r0 + rl) * d + c] = y;
            } else if (c < ldx) {
                out[c] = Half16<WT>::from_float(0.f);
            }
        }
    }
}

// ------------------------------------------------------------------ products

// Pitch (elements) of a normalised input tile in shared memory: rows 64
// bytes apart modulo 128, so the 8 lanes of a B-fragment read phase (2 rows
// x 64 bytes) hit distinct banks.
__host__ __device__ inline int tile_pitch(int kpd) { return kpd % 64 == 0 ? kpd + 32 : kpd; }

// One 1 KB weight chunk against RT = 8*NT input rows.  Weight rows are the
// MMA's M side and input rows its N side (swap-AB), so a single decode row is
// a real m16n8k16 tile.  Lane (g, t) reads its 32 packed bytes (rows g and
// g+8, k = 8t..8t+7) and 16 bytes of each input row at the same k; the two
// k-steps take the halves, so the input fragments follow the weight
// fragments' k permutation and every product pairs the right elements.
template <typename WT, int NT, bool X_SHARED>
__device__ __forceinline__ void product_chunk(const unsigned char* unit, int c, const WT* X, int ldx, int k0,
                                              const bool (&x_ok)[NT], float (&acc)[NT][4]) {
    const int lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;
    const uint4* w = reinterpret_cast<const uint4*>(unit + ((size_t)c * 32 + lane) * 32);
    const uint4 lo = w[0], hi = w[1];
    uint4 B[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const WT* at = X + (size_t)(x_ok[j] ? 8 * j + gq : 0) * ldx + k0 + 8 * tq;
        if (!x_ok[j]) B[j] = make_uint4(0, 0, 0, 0);
        else if constexpr (X_SHARED) B[j] = *reinterpret_cast<const uint4*>(at);
        else B[j] = ld_cg4(at);
    }
    const uint32_t a0[4] = {lo.x, hi.x, lo.y, hi.y};
    const uint32_t a1[4] = {lo.z, hi.z, lo.w, hi.w};
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const uint32_t b0[2] = {B[j].x, B[j].y};
        const uint32_t b1[2] = {B[j].z, B[j].w};
        mma_16816<WT>(acc[j], a0, b0);
        mma_16816<WT>(acc[j], a1, b1);
    }
}

// One 16-row tile over all of K: its units come off the weight stream in
// order, the 8 warps taking alternate chunks of each.  False if a wait gave
// up (the abort word is then raised and the kernel is on its way out).
template <typename WT, int NT, bool X_SHARED>
__device__ bool product_tile(const StepParams& p, Stream& s, int kp, const WT* X, int ldx, int rows_valid,
                             float (&acc)[NT][4]) {
    constexpr int RT = 8 * NT;
    __shared__ int gave_up;
    const int warp = threadIdx.x >> 5, gq = (threadIdx.x & 31) >> 2;
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    bool x_ok[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) x_ok[j] = 8 * j + gq < rows_valid;
    const int chunks = kp / 32;
    for (int c0 = 0; c0 < chunks; c0 += kUnitChunks) {
        const int n = min(kUnitChunks, chunks - c0);
        if (threadIdx.x == 0) gave_up = wait_unit(p, s, s.consumed) ? 0 : 1;
        __syncthreads();
        if (gave_up) return false;
        wait_unit(p, s, s.consumed);  // every thread observes the completed phase
        const unsigned char* unit = s.ring + (size_t)(s.consumed % s.stages) * kUnitBytes;
        for (int c = warp; c < n; c += kWarps)
            product_chunk<WT, NT, X_SHARED>(unit, c, X, ldx, (c0 + c) * 32, x_ok, acc);
        release_unit<RT>(p, s);
    }
    return true;
}

// Folds the 8 warps' K slices into red[16][RT] sums, in a fixed order.
template <int NT>
__device__ __forceinline__ void product_reduce(float* red, const float (&acc)[NT][4]) {
    constexpr int RT = 8 * NT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const int col = 8 * j + 2 * tq;
        red[(warp * 16 + gq) * RT + col] = acc[j][0];
        red[(warp * 16 + gq) * RT + col + 1] = acc[j][1];
        red[(warp * 16 + gq + 8) * RT + col] = acc[j][2];
        red[(warp * 16 + gq + 8) * RT + col + 1] = acc[j][3];
    }
    __syncthreads();
}

__device__ __forceinline__ float product_sum(const float* red, int RT, int nl, int rl) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[(w * 16 + nl) * RT + rl];
    return v;
}

// Work area of a product: [xs: RT x pitch 16-bit][red: 8 x 16 x RT][tile: 16 x RT]
//                         [best values: out_rows][best indices: out_rows]
template <typename WT, int NT>
__device__ void op_product(const StepParams& p, const StepOp& op, int position, Stream& s, unsigned char* work) {
    constexpr int RT = 8 * NT;
    const int pitch = tile_pitch(p.kpd);
    WT* xs = reinterpret_cast<WT*>(work);
    float* red = reinterpret_cast<float*>(work + (size_t)RT * pitch * sizeof(WT));
    const bool normalise = op.gamma != nullptr;
    const int n_tiles = (op.n + 15) / 16;
    const int r_tiles = (p.rows + RT - 1) / RT;
    int cached_tile = -1;

    for (int item = blockIdx.x; item < n_tiles * r_tiles; item += gridDim.x) {
        const int r_tile = item / n_tiles, n_tile = item % n_tiles;
        const int r0 = r_tile * RT, n0 = n_tile * 16;
        const int rows_valid = min(RT, p.rows - r0);
        float acc[NT][4];
        bool ok;
        if (normalise) {
            if (cached_tile != r_tile) {
                __syncthreads();
                layer_norm_tile<WT>(p, op.gamma, op.beta, r0, rows_valid, 1, 0, xs, pitch, nullptr);
                __syncthreads();
                cached_tile = r_tile;
            }
            ok = product_tile<WT, NT, true>(p, s, op.kp, xs, pitch, rows_valid, acc);
        } else {
            const WT* X = static_cast<const WT*>(op.input16) + (size_t)r0 * op.ld_input;
            ok = product_tile<WT, NT, false>(p, s, op.kp, X, op.ld_input, rows_valid, acc);
        }
        if (!ok) return;
        product_reduce<NT>(red, acc);
        for (int o = threadIdx.x; o < 16 * RT; o += kThreads) {
            const int nl = o / RT, rl = o % RT;
            const int n = n0 + nl, r = r0 + rl;
            if (n >= op.n || rl >= rows_valid) continue;
            float v = product_sum(red, RT, nl, rl);
            if (op.bias) v += op.bias[n];
            switch (op.epilogue) {
            case kEpStore:
                static_cast<float*>(op.out)[(size_t)r * op.ld_out + n] = v;
                break;
            case kEpResidual: {
                float* at = static_cast<float*>(op.out) + (size_t)r * op.ld_out + n;
                *at = ld_cg(at) + v;
                break;
            }
            case kEpGelu:
                static_cast<WT*>(op.out)[(size_t)r * op.ld_out + n] = Half16<WT>::from_float(gelu_exact(v));
                break;
            case kEpQkv:
                if (n < p.width) {
                    static_cast<float*>(op.out)[(size_t)r * op.ld_out + n] = v;
                } else {
                    const int which = (n - p.width) / p.width;
                    const int c = n - p.width - which * p.width;
                    const int b = r / p.tokens, t = r % p.tokens;
                    WT* cache = static_cast<WT*>(which == 0 ? op.self_keys : op.self_values);
                    cache[((size_t)b * p.max_positions + position + t) * p.width + c] = Half16<WT>::from_float(v);
                }
                break;
            }
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------- logits

// LN(h) of the sampled rows against the tied token table, with the masked
// argmax folded in: each CTA keeps, per row, the first maximum over the
// columns it produced; the last CTA to finish folds the CTAs' candidates,
// writes each window's sampled id into its next token slot and advances the
// position.
template <typename WT, int NT>
__device__ void op_logits(const StepParams& p, int position, Stream& s, unsigned char* work) {
    constexpr int RT = 8 * NT;
    const int pitch = tile_pitch(p.kpd);
    WT* xs = reinterpret_cast<WT*>(work);
    float* red = reinterpret_cast<float*>(work + (size_t)RT * pitch * sizeof(WT));
    float* tile = red + kWarps * 16 * RT;
    float* best_v = tile + 16 * RT;
    uint32_t* best_i = reinterpret_cast<uint32_t*>(best_v + p.out_rows);
    __shared__ int is_last;

    for (int r = threadIdx.x; r < p.out_rows; r += kThreads) {
        best_v[r] = -INFINITY;
        best_i[r] = kUnchosen;
    }
    const int n_tiles = (p.vocabulary + 15) / 16;
    const int r_tiles = (p.out_rows + RT - 1) / RT;
    int cached_tile = -1;
    __syncthreads();

    for (int item = blockIdx.x; item < n_tiles * r_tiles; item += gridDim.x) {
        const int r_tile = item / n_tiles, n_tile = item % n_tiles;
        const int r0 = r_tile * RT, n0 = n_tile * 16;
        const int rows_valid = min(RT, p.out_rows - r0);
        if (cached_tile != r_tile) {
            __syncthreads();
            layer_norm_tile<WT>(p, p.final_gamma, p.final_beta, r0, rows_valid, p.row_step, p.row_offset, xs, pitch,
                                p.hidden_out);
            __syncthreads();
            cached_tile = r_tile;
        }
        float acc[NT][4];
        if (!product_tile<WT, NT, true>(p, s, p.kpd, xs, pitch, rows_valid, acc)) return;
        product_reduce<NT>(red, acc);
        for (int o = threadIdx.x; o < 16 * RT; o += kThreads) {
            const int nl = o / RT, rl = o % RT;
            const float v = product_sum(red, RT, nl, rl);
            tile[nl * RT + rl] = v;
            const int n = n0 + nl;
            if (p.logits_out && n < p.vocabulary && rl < rows_valid)
                p.logits_out[(size_t)(r0 + rl) * p.vocabulary + n] = v;
        }
        __syncthreads();
        for (int rl = threadIdx.x; rl < rows_valid; rl += kThreads) {
            float bv = best_v[r0 + rl];
            uint32_t bi = best_i[r0 + rl];
            for (int nl = 0; nl < 16; ++nl) {
                const int n = n0 + nl;
                if (n >= p.vocabulary) break;
                if (p.mask && p.mask[n] != 0.f) continue;
                const float v = tile[nl * RT + rl];
                if (candidate_better(v, (uint32_t)n, bv, bi)) { bv = v; bi = (uint32_t)n; }
            }
            best_v[r0 + rl] = bv;
            best_i[r0 + rl] = bi;
        }
        __syncthreads();
    }

    // This CTA's candidates, then the fold by whichever CTA finishes last.
    for (int r = threadIdx.x; r < p.out_rows; r += kThreads) {
        p.candidate_values[(size_t)r * gridDim.x + blockIdx.x] = best_v[r];
        p.candidate_indices[(size_t)r * gridDim.x + blockIdx.x] = best_i[r];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(p.logits_counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rows_per_window = p.out_rows / p.windows;
    for (int r = warp; r < p.out_rows; r += kWarps) {
        float bv = -INFINITY;
        uint32_t bi = kUnchosen;
        for (int c = lane; c < (int)gridDim.x; c += 32) {
            const float v = ld_cg(p.candidate_values + (size_t)r * gridDim.x + c);
            const uint32_t i = ld_cg(p.candidate_indices + (size_t)r * gridDim.x + c);
            if (candidate_better(v, i, bv, bi)) { bv = v; bi = i; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (candidate_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) {
            const uint32_t chosen = bi == kUnchosen ? 0u : bi;  // Argmax.h:190-193
            if (p.row_tokens) p.row_tokens[r] = chosen;
            const int b = r / rows_per_window;
            if (p.write_ring && r % rows_per_window == rows_per_window - 1) {
                p.ring[(size_t)b * p.ring_stride + position + p.tokens] = chosen;
                if (p.stop_enabled && chosen == p.stop_token) p.ended[b] = 1;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (p.stop_enabled) {
            int all = 1;
            for (int b = 0; b < p.windows; ++b) all &= p.ended[b] ? 1 : 0;
            if (all) atomicExch(p.state + kAllEnded, 1);
        }
        atomicAdd(p.state + kStepsDone, 1);
        atomicAdd(p.state + kPosition, p.tokens);
        atomicExch(p.logits_counter, 0u);
        __threadfence();
    }
}

// ----------------------------------------------------------------- attention

// Scores of keys [k0, k1) against q (in shared, pre-scaled), into scores[];
// returns this thread's maximum.
template <typename WT, bool READ_ONLY>
__device__ __forceinline__ float attention_scores(const float* q, const WT* K, long long key_stride, int D, int k0,
                                                  int n, float* scores) {
    float local_max = -INFINITY;
    for (int j = threadIdx.x; j < n; j += kThreads) {
        const WT* krow = K + (size_t)(k0 + j) * key_stride;
        float s = 0.f;
        if (D % 8 == 0) {
            for (int c = 0; c < D; c += 8) {
                const uint4 u = READ_ONLY ? load_stream(krow + c) : ld_cg4(krow + c);
                const float2 f0 = Half16<WT>::pair_to_float2(u.x), f1 = Half16<WT>::pair_to_float2(u.y);
                const float2 f2 = Half16<WT>::pair_to_float2(u.z), f3 = Half16<WT>::pair_to_float2(u.w);
                s += q[c] * f0.x + q[c + 1] * f0.y + q[c + 2] * f1.x + q[c + 3] * f1.y + q[c + 4] * f2.x +
                     q[c + 5] * f2.y + q[c + 6] * f3.x + q[c + 7] * f3.y;
            }
        } else {
            for (int c = 0; c < D; ++c)
                s += q[c] * bits_to_float<WT>(READ_ONLY ? ld_nc_u16(krow + c) : ld_cg_u16(krow + c));
        }
        scores[j] = s;
        local_max = fmaxf(local_max, s);
    }
    return local_max;
}

// sum_j p_j V[k0 + j] over the keys into result[0..D).  With D a multiple
// of 8, thread (group, piece) reads 16 bytes of a value row per key and the
// 256/(D/8) key groups fold in shared memory (fold holds 2048 floats).
template <typename WT, bool READ_ONLY>
__device__ __forceinline__ void attention_values(const float* scores, const WT* V, long long key_stride, int D,
                                                 int k0, int n, float* fold, float* result) {
    if (D % 8 == 0) {
        const int pieces = D / 8;
        const int groups = kThreads / pieces;
        const int piece = threadIdx.x % pieces, g = threadIdx.x / pieces;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (g < groups) {
            for (int j = g; j < n; j += groups) {
                const WT* at = V + (size_t)(k0 + j) * key_stride + piece * 8;
                const uint4 u = READ_ONLY ? load_stream(at) : ld_cg4(at);
                const float w = scores[j];
                const float2 f0 = Half16<WT>::pair_to_float2(u.x), f1 = Half16<WT>::pair_to_float2(u.y);
                const float2 f2 = Half16<WT>::pair_to_float2(u.z), f3 = Half16<WT>::pair_to_float2(u.w);
                acc[0] += w * f0.x; acc[1] += w * f0.y; acc[2] += w * f1.x; acc[3] += w * f1.y;
                acc[4] += w * f2.x; acc[5] += w * f2.y; acc[6] += w * f3.x; acc[7] += w * f3.y;
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) fold[g * D + piece * 8 + e] = acc[e];
        }
        __syncthreads();
        if (threadIdx.x < D) {
            float o = 0.f;
            for (int gg = 0; gg < groups; ++gg) o += fold[gg * D + threadIdx.x];
            result[threadIdx.x] = o;
        }
    } else {
        const int groups = kThreads / D;
        const int c = threadIdx.x % D, g = threadIdx.x / D;
        float acc = 0.f;
        if (g < groups)
            for (int j = g; j < n; j += groups) {
                const WT* at = V + (size_t)(k0 + j) * key_stride + c;
                acc += scores[j] * bits_to_float<WT>(READ_ONLY ? ld_nc_u16(at) : ld_cg_u16(at));
            }
        if (g < groups) fold[g * D + c] = acc;
        __syncthreads();
        if (threadIdx.x < D) {
            float o = 0.f;
            for (int gg = 0; gg < groups; ++gg) o += fold[gg * D + threadIdx.x];
            result[threadIdx.x] = o;
        }
    }
    __syncthreads();
}

// Shared memory of attention: [q: 64][scratch: 8][fold: 2048][result: 64][scores: ...]
constexpr int kFold = 2048;
constexpr int kAttentionFixed = 64 + 8 + kFold + 64;

// Self-attention of row (b, t) and head h over keys 0..position+t: one item.
template <typename WT>
__device__ void op_self_attention(const StepParams& p, const StepOp& op, int position, unsigned char* smem) {
    float* q = reinterpret_cast<float*>(smem);
    float* scratch = q + 64;
    float* fold = scratch + 8;
    float* result = fold + kFold;
    float* scores = result + 64;
    const int D = p.head_width;
    for (int item = blockIdx.x; item < p.rows * p.heads; item += gridDim.x) {
        const int r = item / p.heads, head = item % p.heads;
        const int b = r / p.tokens, t = r % p.tokens;
        const int keys = position + t + 1;
        __syncthreads();
        for (int c = threadIdx.x; c < D; c += kThreads) q[c] = ld_cg(p.q + (size_t)r * p.width + head * D + c) * p.scale;
        __syncthreads();
        const WT* K = static_cast<const WT*>(op.keys) + (size_t)b * op.window_stride + (size_t)head * D;
        const WT* V = static_cast<const WT*>(op.values) + (size_t)b * op.window_stride + (size_t)head * D;
        const float m = block_max(attention_scores<WT, false>(q, K, op.key_stride, D, 0, keys, scores), scratch);
        float local = 0.f;
        for (int j = threadIdx.x; j < keys; j += kThreads) {
            const float e = __expf(scores[j] - m);
            scores[j] = e;
            local += e;
        }
        const float l = block_sum(local, scratch);
        attention_values<WT, false>(scores, V, op.key_stride, D, 0, keys, fold, result);
        WT* out = static_cast<WT*>(p.attn16) + (size_t)r * p.kpd + head * D;
        for (int c = threadIdx.x; c < D; c += kThreads) out[c] = Half16<WT>::from_float(result[c] / l);
    }
}

// Cross-attention item (row, head, split): the split's max, sum and
// unnormalised row; the last split of a (row, head) to finish joins them the
// way a split softmax joins (SingleQueryAttention.h:11-37) and adds the
// v_proj bias (the weights sum to one, so the bias passes through).
template <typename WT>
__device__ void op_cross_attention(const StepParams& p, const StepOp& op, unsigned char* smem) {
    float* q = reinterpret_cast<float*>(smem);
    float* scratch = q + 64;
    float* fold = scratch + 8;
    float* result = fold + kFold;
    float* scores = result + 64;
    __shared__ int is_last;
    const int D = p.head_width;
    const int S = op.splits;
    for (int item = blockIdx.x; item < p.rows * p.heads * S; item += gridDim.x) {
        const int split = item % S;
        const int head = (item / S) % p.heads;
        const int r = item / (S * p.heads);
        const int b = r / p.tokens;
        const int k0 = split * op.chunk;
        const int n = min(op.key_count, k0 + op.chunk) - k0;
        float* out = p.partial + (((size_t)r * p.heads + head) * S + split) * (D + 2);
        __syncthreads();
        if (n <= 0) {
            for (int c = threadIdx.x; c < D + 2; c += kThreads) out[c] = c == 0 ? -INFINITY : 0.f;
        } else {
            for (int c = threadIdx.x; c < D; c += kThreads)
                q[c] = ld_cg(p.q + (size_t)r * p.width + head * D + c) * p.scale;
            __syncthreads();
            const WT* K = static_cast<const WT*>(op.keys) + (size_t)b * op.window_stride + (size_t)head * D;
            const WT* V = static_cast<const WT*>(op.values) + (size_t)b * op.window_stride + (size_t)head * D;
            const float m = block_max(attention_scores<WT, true>(q, K, op.key_stride, D, k0, n, scores), scratch);
            float local = 0.f;
            for (int j = threadIdx.x; j < n; j += kThreads) {
                const float e = __expf(scores[j] - m);
                scores[j] = e;
                local += e;
            }
            const float l = block_sum(local, scratch);
            attention_values<WT, true>(scores, V, op.key_stride, D, k0, n, fold, result);
            for (int c = threadIdx.x; c < D; c += kThreads) out[2 + c] = result[c];
            if (threadIdx.x == 0) {
                out[0] = m;
                out[1] = l;
            }
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned* counter = p.combine_counters + (size_t)r * p.heads + head;
            is_last = atomicAdd(counter, 1u) == (unsigned)(S - 1);
            if (is_last) atomicExch(counter, 0u);
        }
        __syncthreads();
        if (!is_last) continue;
        __threadfence();
        const float* part = p.partial + ((size_t)r * p.heads + head) * S * (D + 2);
        // Every thread reads the splits' maxima; threads < D then fold a channel.
        float mx = -INFINITY;
        for (int s = 0; s < S; ++s) mx = fmaxf(mx, ld_cg(part + (size_t)s * (D + 2)));
        if (threadIdx.x < D) {
            float l = 0.f, o = 0.f;
            for (int s = 0; s < S; ++s) {
                const float ms = ld_cg(part + (size_t)s * (D + 2));
                if (ms == -INFINITY) continue;
                const float f = __expf(ms - mx);
                l += ld_cg(part + (size_t)s * (D + 2) + 1) * f;
                o += ld_cg(part + (size_t)s * (D + 2) + 2 + threadIdx.x) * f;
            }
            float y = o / l;
            if (op.value_bias) y += op.value_bias[head * D + threadIdx.x];
            static_cast<WT*>(p.attn16)[(size_t)r * p.kpd + head * D + threadIdx.x] = Half16<WT>::from_float(y);
        }
    }
}

// -------------------------------------------------------------- the kernel

template <int NT> struct StreamStages { static constexpr int value = NT <= 2 ? 4 : 3; };

// Thread 0, on the way out: no bulk copy may still be landing in shared
// memory once the CTA exits, so wait (bounded) for every unit issued.
__device__ void drain_stream(const StepParams& p, Stream& s) {
    if (threadIdx.x == 0)
        for (unsigned long long i = s.consumed; i < s.issued; ++i)
            if (!wait_unit(p, s, i)) break;
    __syncthreads();
}

template <typename WT, int NT>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(StepParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int RT = 8 * NT;
    Stream s;
    s.stages = StreamStages<NT>::value;
    s.ring = smem;
    s.full = reinterpret_cast<uint64_t*>(smem + (size_t)s.stages * kUnitBytes);
    unsigned char* work = smem + (size_t)s.stages * kUnitBytes + 128;
    s.consumed = 0;
    s.issued = 0;
    s.cursor = Cursor{0, 0, (int)blockIdx.x, 0};
    if (threadIdx.x == 0) {
        for (int i = 0; i < s.stages; ++i)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_address(s.full + i)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) issue_ahead<RT>(p, s);

    unsigned epoch = 0;
    const bool stamp = p.profile != nullptr && blockIdx.x == 0 && threadIdx.x == 0;
    for (int step = 0; step < p.steps; ++step) {
        const int position = ld_volatile(p.state + kPosition);
        if (stamp && step == 0) p.profile[0] = global_ns();
        for (int i = 0; i < p.n_ops; ++i) {
            const StepOp& op = p.ops[i];
            switch (op.kind) {
            case kOpEmbed: op_embed<WT>(p, position); break;
            case kOpProduct: op_product<WT, NT>(p, op, position, s, work); break;
            case kOpSelfAttention: op_self_attention<WT>(p, op, position, work); break;
            case kOpCrossAttention: op_cross_attention<WT>(p, op, work); break;
            case kOpLogits: op_logits<WT, NT>(p, position, s, work); break;
            }
            if (!grid_barrier(p.barrier, epoch, p.state)) {
                drain_stream(p, s);
                return;
            }
            if (stamp && step == 0) p.profile[i + 1] = global_ns();
        }
        if (p.stop_enabled && ld_volatile(p.state + kAllEnded)) break;
    }
    drain_stream(p, s);
}

template <typename WT, int NT>
size_t shared_bytes(const StepParams& p, int max_chunk) {
    constexpr int RT = 8 * NT;
    const size_t product = (size_t)RT * tile_pitch(p.kpd) * sizeof(WT) +
                           sizeof(float) * (kWarps * 16 * RT + 16 * RT) + (size_t)p.out_rows * 8;
    const size_t attention = sizeof(float) * (kAttentionFixed + std::max(max_chunk, p.max_positions));
    const size_t work = (std::max(product, attention) + 127) / 128 * 128;
    return (size_t)StreamStages<NT>::value * kUnitBytes + 128 + work;
}

template <typename WT, int NT>
void launch_typed(const StepParams& p, int max_chunk, int grid, cudaStream_t stream) {
    const size_t smem = shared_bytes<WT, NT>(p, max_chunk);
    auto kernel = decode_kernel<WT, NT>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) throw std::runtime_error(std::string("decode kernel shared memory: ") + cudaGetErrorString(e));
    StepParams copy = p;
    void* args[] = {&copy};
    e = cudaLaunchCooperativeKernel((const void*)kernel, grid, kThreads, args, smem, stream);
    if (e != cudaSuccess) throw std::runtime_error(std::string("decode kernel launch: ") + cudaGetErrorString(e));
}

template <typename WT, int NT>
int occupancy_typed(const StepParams& p, int max_chunk) {
    const size_t smem = shared_bytes<WT, NT>(p, max_chunk);
    auto kernel = decode_kernel<WT, NT>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, kThreads, smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return blocks;
}

// Input rows per tile: 8, 16, or 32 (more rows run as several tiles).
inline int tile_columns(const StepParams& p) {
    const int rows = std::max(p.rows, p.out_rows);
    return rows <= 8 ? 1 : (rows <= 16 ? 2 : 4);
}

template <typename WT>
void launch_rows(const StepParams& p, int max_chunk, int grid, cudaStream_t stream) {
    switch (tile_columns(p)) {
    case 1: launch_typed<WT, 1>(p, max_chunk, grid, stream); break;
    case 2: launch_typed<WT, 2>(p, max_chunk, grid, stream); break;
    default: launch_typed<WT, 4>(p, max_chunk, grid, stream); break;
    }
}

template <typename WT>
int occupancy_rows(const StepParams& p, int max_chunk) {
    switch (tile_columns(p)) {
    case 1: return occupancy_typed<WT, 1>(p, max_chunk);
    case 2: return occupancy_typed<WT, 2>(p, max_chunk);
    default: return occupancy_typed<WT, 4>(p, max_chunk);
    }
}

}  // namespace

int decode_blocks_per_sm(bool half, const StepParams& p, int max_chunk) {
    return half ? occupancy_rows<__half>(p, max_chunk) : occupancy_rows<__nv_bfloat16>(p, max_chunk);
}

void launch_decode(bool half, const StepParams& p, int max_chunk, int grid, cudaStream_t stream) {
    if (p.width > 32 * kNormMaxPerLane) throw std::invalid_argument("widths above 1536 are not supported");
    if (p.head_width > 64) throw std::invalid_argument("heads wider than 64 are not supported");
    if (half) launch_rows<__half>(p, max_chunk, grid, stream);
    else launch_rows<__nv_bfloat16>(p, max_chunk, grid, stream);
}

}  // namespace wsp
