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
#include "umma.cuh"

#include <type_traits>
#include "step_launch.h"

#include <algorithm>
#include <stdexcept>
#include <string>

namespace wsp {
namespace {

// Consumer warps of the decode kernel: 7, so that with the producer warp a
// CTA is 8 warps -- two per SM sub-partition, each thread keeping the full
// register budget.
constexpr int kWarps = kStepWarps;
constexpr int kThreads = 32 * kWarps;

// ------------------------------------------------------------ memory access

// Data another CTA wrote inside the launch is read through L2 (ld.global.cg:
// never a stale L1 line); the grid barrier orders it.  Weights, biases and
// the cross caches are read-only for the whole launch (ld.global.nc).  The
// compiler's own load builtins keep the loads free to be batched.
__device__ __forceinline__ uint4 ld_cg4(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ uint32_t ld_cg(const uint32_t* p) { return __ldcg(reinterpret_cast<const unsigned int*>(p)); }
__device__ __forceinline__ unsigned short ld_cg_u16(const void* p) {
    return __ldcg(reinterpret_cast<const unsigned short*>(p));
}
__device__ __forceinline__ unsigned short ld_nc_u16(const void* p) {
    return __ldg(reinterpret_cast<const unsigned short*>(p));
}
__device__ __forceinline__ uint4 ld_nc4(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
// The CTA is 8 consumer warps, which run the ops, and one producer warp,
// which only streams weights into the shared-memory ring.  The consumers
// synchronise among themselves on named barrier 1.
constexpr int kConsumers = kThreads;
constexpr int kBlockThreads = kThreads + 32;

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;\n" ::"n"(kConsumers) : "memory"); }

__device__ __forceinline__ float consumer_sum(float v, float* scratch) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    consumer_sync();
    if (lane == 0) scratch[warp] = v;
    consumer_sync();
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) total += scratch[w];
    return total;
}

// consumer_sum for a scratch array no thread can still be reading (the
// caller alternates arrays between barriers): one CTA barrier instead of two.
__device__ __forceinline__ float consumer_sum_fresh(float v, float* scratch) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = v;
    consumer_sync();
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) total += scratch[w];
    return total;
}

__device__ __forceinline__ float consumer_max(float v, float* scratch) {
    v = warp_max(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    consumer_sync();
    if (lane == 0) scratch[warp] = v;
    consumer_sync();
    float best = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) best = fmaxf(best, scratch[w]);
    return best;
}

__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// Element (row r, column c) of a 16-bit activation matrix with row pitch ld:
// row-major, or the tensor-core block layout (act_offset) when p.umma.
__device__ __forceinline__ size_t act_index(const StepParams& p, int r, int c, int ld) {
    return p.umma ? act_offset(r, c, p.act_rows) : (size_t)r * ld + c;
}

// The 16-bit activations a product reads (normalised rows, attended rows,
// GELU outputs) carry two planes: hi = the value rounded to 16 bits, and lo
// = the rest (value - hi) rounded again, act_rows * ld elements past hi in
// the same layout.  A product sums W . hi + W . lo, two tensor-core products
// into one fp32 accumulator, so its input carries about twice the 16-bit
// precision (the rounding of a bf16 activation would otherwise dominate the
// error against fp32 arithmetic).  Tiles in shared memory keep the same two
// planes, `lo` elements apart.
__device__ __forceinline__ size_t lo_plane(const StepParams& p, int ld) { return (size_t)p.act_rows * ld; }

template <typename WT>
__device__ __forceinline__ void store_split(WT* hi, size_t lo, float v) {
    const WT h = Half16<WT>::from_float(v);
    hi[0] = h;
    hi[lo] = Half16<WT>::from_float(v - Half16<WT>::to_float(h));
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Adds one to a gpu-scope counter with acquire-release semantics and returns
// the old value: after a CTA barrier, it releases everything the CTA wrote
// before it and, for the arrival that sees the others', acquires what they
// released -- one round trip, no separate fences.
__device__ __forceinline__ unsigned arrive_acq_rel(unsigned* counter) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;\n" : "=r"(old) : "l"(counter) : "memory");
    return old;
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Section timers for measurement: CTA 0, thread 0 accumulates clock64
// cycles per section of a launch into profile[kTraceBase + section] when a
// profile buffer is given.
enum TraceSection : int { kTrWait = 0, kTrCompute, kTrBarrier, kTrEpilogue, kTrNorm, kTrAttention, kTrOther,
                          kTrQuery, kTrJoin, kTrOutProj, kTrSelf, kTrLogits, kTrNormLoad, kTrNormRest, kTrLogitsTiles,
                          kTrLogitsFold, kTrSections };
constexpr int kTraceBase = 512;
__shared__ unsigned long long trace_cycles[kTrSections];

struct Trace {
    bool on;
    long long start;
    __device__ __forceinline__ void begin() { if (on) start = clock64(); }
    __device__ __forceinline__ void end(int section) {
        if (on) trace_cycles[section] += (unsigned long long)(clock64() - start);
    }
};
__device__ __forceinline__ Trace trace_of(const unsigned long long* profile) {
    Trace t;
    t.on = profile != nullptr && blockIdx.x == 0 && threadIdx.x == 0;
    t.start = 0;
    return t;
}

// CTA 0's thread 0 adds its section cycles into profile[kTraceBase ...].
__device__ __forceinline__ void trace_flush(const StepParams& p) {
    if (p.profile != nullptr && blockIdx.x == 0 && threadIdx.x == 0)
        for (int i = 0; i < kTrSections; ++i) p.profile[kTraceBase + i] += trace_cycles[i];
}

template <typename WT>
__device__ __forceinline__ float bits_to_float(unsigned short b) {
    return Half16<WT>::to_float(*reinterpret_cast<const WT*>(&b));
}

// -------------------------------------------------------------- grid barrier

constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;  // 2 s
constexpr unsigned long long kAbortLookNs = 50000ull;          // 50 us

// A monotonic arrival counter: each CTA adds one with release semantics and
// polls with acquire loads, nothing else in flight, until every CTA has
// arrived `epoch` times.  A wait that gives up anywhere in the kernel
// (record_timeout) also adds kAbortBias to the counter, so every CTA polling
// it sees the failure on the same load that would have seen the barrier
// complete -- no second word to read per poll or per barrier.  The poll
// reads the clock every 32 loads and gives up after kWaitTimeoutNs: it
// records kErrBarrierTimeout and the kernel returns.  (Arrivals per launch
// stay far below the bias: steps x ops x CTAs < 2^30.)
constexpr unsigned kAbortBias = 1u << 30;

// Records the first wait that gave up: its kind, CTA and op/unit index; then
// raises the abort word (read by long ring waits) and the barrier's bias.
__device__ __forceinline__ void record_timeout(const StepParams& p, int kind, long long where) {
    atomicOr(p.state + kError, kErrBarrierTimeout);
    if (atomicCAS(p.state + kFailKind, 0, kind) == 0) {
        p.state[kFailCta] = (int)blockIdx.x;
        p.state[kFailWhere] = (int)where;
    }
    // The first to give up adds the bias, once: more would wrap the counter.
    if (atomicExch(p.state + kAbort, 1) == 0) atomicAdd(p.barrier, kAbortBias);
}

// The op list is read-only for the whole launch, and a grid barrier's
// acquire leaves nothing of it in L1: read from global memory after the
// barrier, an op's fields would cost a round trip to L2 before its first
// load of data could issue.  So while thread 0 waits at the barrier, threads
// 1.. copy the next op into a shared-memory slot with non-coherent loads,
// and the op after the barrier reads its fields from there.
constexpr int kOpWords = (int)(sizeof(StepOp) / sizeof(unsigned long long));
static_assert(sizeof(StepOp) % sizeof(unsigned long long) == 0, "StepOp copies as 8-byte words");
static_assert(kOpWords < kConsumers, "a consumer thread a word of the op");
__device__ __forceinline__ void copy_op(const StepOp* from, StepOp* to, int word) {
    if (word >= 0 && word < kOpWords)
        reinterpret_cast<unsigned long long*>(to)[word] =
            __ldg(reinterpret_cast<const unsigned long long*>(from) + word);
}

__device__ bool grid_barrier(const StepParams& p, unsigned& epoch, const StepOp* next, StepOp* next_slot) {
    __shared__ int aborted;
    consumer_sync();
    ++epoch;
    if (threadIdx.x != 0) copy_op(next, next_slot, (int)threadIdx.x - 1);
    if (threadIdx.x == 0) {
        asm volatile("red.release.gpu.global.add.u32 [%0], %1;\n" ::"l"(p.barrier), "r"(1u) : "memory");
        const unsigned target = epoch * gridDim.x;
        unsigned seen = ld_acquire(p.barrier);
        if (seen < target) {
            const unsigned long long start = global_ns();
            for (unsigned spin = 1; (seen = ld_acquire(p.barrier)) < target; ++spin) {
                if ((spin & 31) == 0 && global_ns() - start > kWaitTimeoutNs) {
                    record_timeout(p, kWaitGrid, (long long)epoch);
                    seen = kAbortBias;
                    break;
                }
            }
        }
        aborted = seen >= kAbortBias;
    }
    consumer_sync();
    return aborted == 0;
}

// ------------------------------------------------------------ weight stream

// Weight tiles stream through a ring of shared-memory stages.  The producer
// warp walks the CTA's schedule (built on the host, schedule.h) -- every
// unit of weights the CTA's ops consume in a step, in order, step after step
// -- and fills stage u % S with unit u by one cp.async.bulk copy that
// completes full[u % S], once the consumers have released unit u - S
// through empty[u % S].  The consumers wait on full[], read, and release
// warp by warp, so no CTA-wide sync is spent per unit, and the next op's
// first units land while this op and the grid barrier run.

// Ring positions: unit u sits in stage u % stages, round u / stages.  The
// division is by a launch constant (2 or more stages), so it is a
// multiply-high by its reciprocal, ceil(2^32 / stages): exact for u < 2^32 /
// stages (a launch streams a few million units at most), where a 64-bit % or
// / by a runtime value would be a software routine of a hundred-odd
// instructions on every wait and release.
struct RingDivisor {
    uint32_t count, magic;
    __device__ __forceinline__ void set(int n) {
        count = (uint32_t)n;
        magic = (uint32_t)(0xFFFFFFFFull / (unsigned long long)n) + 1u;
    }
    __device__ __forceinline__ uint32_t round(unsigned long long u) const { return __umulhi((uint32_t)u, magic); }
    __device__ __forceinline__ uint32_t slot(unsigned long long u) const { return (uint32_t)u - round(u) * count; }
};

struct Stream {
    unsigned char* ring;          // stages x stage_bytes
    uint64_t* full;               // per stage: the unit landed (tx bytes)
    uint64_t* empty;              // per stage: the 8 consumer warps released it
    int stages;
    RingDivisor div;              // stage and round of a unit index
    int stage_bytes;
    unsigned long long next;      // the next unit this CTA's consumers reach
    volatile unsigned long long* armed;  // units the producer has armed full[] for
};

__device__ __forceinline__ bool try_parity(uint64_t* bar, uint32_t parity) {
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

// Waits for the phase of `parity` to complete, for at most kWaitTimeoutNs;
// gives up early when *stop is raised.  On a timeout it records
// kErrBarrierTimeout and raises the abort word.
__device__ bool wait_parity(const StepParams& p, uint64_t* bar, uint32_t parity, const volatile int* stop, int kind,
                            unsigned long long index) {
    if (try_parity(bar, parity)) return true;
    const unsigned long long start = global_ns();
    for (unsigned spin = 1; !try_parity(bar, parity); ++spin) {
        if (stop && *stop) return false;
        if ((spin & 15) != 0) continue;
        const unsigned long long waited = global_ns() - start;
        if (waited > kWaitTimeoutNs) {
            record_timeout(p, kind, (long long)index);
            return false;
        }
        // A wait this long may be one another wait's failure left
        // unanswered: look at the abort word (a global load, so never in a
        // short wait).  The producer's final drain still waits for its copies.
        if (waited > kAbortLookNs && kind != kWaitDrain && ld_volatile(p.state + kAbort)) return false;
    }
    return true;
}

// Consumers: unit `index` landed.  A wait that gave up (the abort word is
// then raised) returns the stage all the same, so every warp keeps the same
// path to the next grid barrier, where the kernel leaves.
__device__ __forceinline__ const unsigned char* unit_at(const StepParams& p, const Stream& s, unsigned long long index) {
    Trace tr = trace_of(p.profile);
    tr.begin();
    const int stage = (int)s.div.slot(index);
    wait_parity(p, s.full + stage, s.div.round(index) & 1u, nullptr, kWaitUnit, index);
    tr.end(kTrWait);
    return s.ring + (size_t)stage * s.stage_bytes;
}

// A warp that owns whole units (the logits) skips the units between its own,
// so it may reach unit `index` before unit index - stages, which shares the
// stage, has landed; the stage's parity would then read as index's.  Once the
// producer has armed full[] for `index` (after index - stages was released,
// so after it landed), the parity names `index` alone: wait for that first.
__device__ __forceinline__ const unsigned char* owned_unit_at(const StepParams& p, const Stream& s,
                                                              unsigned long long index) {
    if (*s.armed <= index) {
        Trace tr = trace_of(p.profile);
        tr.begin();
        const unsigned long long start = global_ns();
        while (*s.armed <= index) {
            if (global_ns() - start > kWaitTimeoutNs) {
                record_timeout(p, kWaitArmed, (long long)index);
                break;
            }
        }
        tr.end(kTrWait);
    }
    __threadfence_block();
    return unit_at(p, s, index);
}

// Consumers: this warp is done with unit `index` (its share of it, or the
// whole of it when the warp owns the unit: count 8).
__device__ __forceinline__ void release_at(const Stream& s, unsigned long long index, unsigned count = 1) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0)
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_address(s.empty + s.div.slot(index))),
                     "r"(count)
                     : "memory");
}

// The shared-unit pattern: every warp reads the next unit, then releases it.
__device__ __forceinline__ const unsigned char* acquire_unit(const StepParams& p, const Stream& s) {
    return unit_at(p, s, s.next);
}
__device__ __forceinline__ void release_unit(Stream& s) {
    release_at(s, s.next);
    ++s.next;
}

// An L2 prefetch of [ptr, ptr + bytes): a bulk prefetch (no data comes back
// to the SM, nothing waits for it), which wants 16-byte alignment: the start
// is rounded down to 16 bytes (never below its allocation, whose start is
// aligned) and the end down as well.
__device__ __forceinline__ void prefetch_l2(const void* ptr, unsigned long long bytes) {
    const unsigned long long start = reinterpret_cast<unsigned long long>(ptr) & ~15ull;
    const unsigned long long end = (reinterpret_cast<unsigned long long>(ptr) + bytes) & ~15ull;
    if (end > start)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(start), "r"((unsigned)(end - start))
                     : "memory");
}

// The producer warp's lane 0: the CTA's schedule for every step, then a
// wait for every copy still landing, so none outlives the CTA.
__device__ void produce(const StepParams& p, Stream& s, const volatile int* stop) {
    const unsigned first = __ldg(p.schedule_offsets + blockIdx.x);
    const unsigned count = __ldg(p.schedule_offsets + blockIdx.x + 1) - first;
    const ulonglong2* schedule = reinterpret_cast<const ulonglong2*>(p.schedule) + first;
    unsigned long long u = 0;
    bool go = count > 0;
    for (int step = 0; go && step < p.steps; ++step) {
        for (unsigned i = 0; i < count; ++i) {
            const ulonglong2 e = __ldg(schedule + i);
            if (e.y & kPrefetchOnly) {
                // Not a unit: an L2 prefetch of data an op ahead reads straight
                // from memory (its parameters, a fused out-projection's columns).
                prefetch_l2(reinterpret_cast<const void*>(e.x), (unsigned)e.y);
                continue;
            }
            const int stage = (int)s.div.slot(u);
            if (u >= (unsigned long long)s.stages &&
                !wait_parity(p, s.empty + stage, (s.div.round(u) - 1u) & 1u, stop, kWaitEmpty, u)) {
                go = false;
                break;
            }
            const uint32_t bar = smem_address(s.full + stage);
            const uint32_t dst = smem_address(s.ring + (size_t)stage * s.stage_bytes);
            const unsigned bytes = (unsigned)e.y;
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
                "l"(e.x), "r"(bytes), "r"(bar)
                : "memory");
            __threadfence_block();
            *s.armed = u + 1;
            ++u;
        }
    }
    const unsigned long long stages = (unsigned long long)s.stages;
    for (unsigned long long v = u > stages ? u - stages : 0; v < u; ++v)
        if (!wait_parity(p, s.full + s.div.slot(v), s.div.round(v) & 1u, nullptr, kWaitDrain, v)) break;
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
        // The token table is laid out for the logits' products: fragment-packed,
        // or the tcgen05 tiles with the tensor-core products.
        for (int c = threadIdx.x; c < p.width; c += kThreads)
            out[c] = Half16<WT>::to_float(table[p.umma ? umma_offset((int)token, c, p.kpd / 64)
                                                       : packed_offset((int)token, c, chunks)]) +
                     pos[c];
    }
}

// ------------------------------------------------------- layer-norm prologue

constexpr int kNormMaxPerLane = 48;  // widths up to 1536

// Terms added to a LayerNorm's input rows before normalising: the bias and
// count partial rows (stride floats apart, row-major [R][d] each), summed in
// order; sum_out, when given, receives the sums (the new residual rows).
struct Addends {
    const float* base = nullptr;
    int count = 0;
    long long stride = 0;
    const float* bias = nullptr;
    float* sum_out = nullptr;
    int tile_rows = 0;  // > 0: a tensor-core product's split partials (StepOp::addend_tile_rows)
};

// v[i] (element c0 + i*step of row `row`, i < N, columns below d) plus the
// addends, every load of a batch of four partial rows in flight at once.
template <int N>
__device__ __forceinline__ void add_addends(const Addends& a, size_t row, int d, int c0, int step, float (&v)[N]) {
    const float* rowp = a.base + row * d;
    // Eight partial rows a batch for a few values a thread (every load of a
    // base.en-sized op in flight at once); one for many (a row's own loads
    // are then plenty in flight).  The bias and the first batch are loaded
    // before the first addition, which waits for the caller's loads of v:
    // one round trip to L2 for the row and its addends, not two.
    constexpr int kBatch = N <= 8 ? 8 : 1;
    float bias[N];
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const int c = c0 + i * step;
        bias[i] = c < d ? __ldg(a.bias + c) : 0.f;
    }
    if (a.tile_rows > 0) {
        // A tensor-core product's split partials: element (row, c) of split j
        // at j * stride + ((c / 128) * tile_rows + row) * 128 + c % 128.
        // The splits sum in order from zero, the bias is added to that sum
        // and the result to the row -- the product's join (its sum plus
        // bias, added to the residual row), bit for bit.
        float sum[N];
        int at[N];
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const int c = c0 + i * step;
            sum[i] = 0.f;
            at[i] = ((c >> 7) * a.tile_rows + (int)row) * 128 + (c & 127);
        }
        for (int j0 = 0; j0 < a.count; j0 += kBatch) {
            float t[kBatch][N];
#pragma unroll
            for (int jj = 0; jj < kBatch; ++jj)
#pragma unroll
                for (int i = 0; i < N; ++i)
                    t[jj][i] = j0 + jj < a.count && c0 + i * step < d
                                   ? ld_cg(a.base + (size_t)(j0 + jj) * a.stride + at[i])
                                   : 0.f;
#pragma unroll
            for (int jj = 0; jj < kBatch; ++jj)
                if (j0 + jj < a.count) {
#pragma unroll
                    for (int i = 0; i < N; ++i) sum[i] += t[jj][i];
                }
        }
#pragma unroll
        for (int i = 0; i < N; ++i)
            if (c0 + i * step < d) v[i] += sum[i] + bias[i];
        return;
    }
    for (int j0 = 0; j0 < a.count; j0 += kBatch) {
        float t[kBatch][N];
#pragma unroll
        for (int jj = 0; jj < kBatch; ++jj)
#pragma unroll
            for (int i = 0; i < N; ++i) {
                const int c = c0 + i * step;
                t[jj][i] = j0 + jj < a.count && c < d ? ld_cg(rowp + (size_t)(j0 + jj) * a.stride + c) : 0.f;
            }
        if (j0 == 0) {
#pragma unroll
            for (int i = 0; i < N; ++i)
                if (c0 + i * step < d) v[i] += bias[i];
        }
#pragma unroll
        for (int jj = 0; jj < kBatch; ++jj)
#pragma unroll
            for (int i = 0; i < N; ++i) v[i] += t[jj][i];
    }
    if (a.count <= 0) {
#pragma unroll
        for (int i = 0; i < N; ++i)
            if (c0 + i * step < d) v[i] += bias[i];
    }
}

// LayerNorm of rows_in_tile rows of h into the 16-bit tile xs [rows][ldx]
// (hi) and xs + lo (lo): output row rl reads h row (r0 + rl)*row_step +
// row_offset.  One warp a row,
// the row in registers: the mean, then the centred variance, as
// LayerNorm.h:19-98 does.  hidden_out, when given, receives the fp32 rows.
// With addends, each row is first input + bias + the partial rows (the
// residual additions of a fused out-projection, Decoder.cpp:80-104).
template <typename WT>
__device__ void layer_norm_tile(const StepParams& p, const float* input, const float* gamma, const float* beta,
                                int r0, int rows_in_tile, int row_step, int row_offset, WT* xs, int ldx,
                                size_t lo, float* hidden_out, const Addends& add = Addends()) {
    const int d = p.width;
    if (rows_in_tile <= 2) {
        // A row or two: the whole CTA on each row, every load of the row,
        // the gains and the offsets in flight at once.  The mean and the
        // centred sum reduce through two scratch arrays, one barrier each:
        // a thread that passes one reduction's barrier knows every thread
        // has finished reading the other array (callers sync between calls).
        __shared__ float scratch[2][kWarps];
        constexpr int kPer = (1536 + kThreads - 1) / kThreads;
        for (int rl = 0; rl < rows_in_tile; ++rl) {
            Trace trl = trace_of(p.profile);
            trl.begin();
            const size_t row = (size_t)(r0 + rl) * row_step + row_offset;
            const float* x = input + row * d;
            float v[kPer], g[kPer], b[kPer];
#pragma unroll
            for (int i = 0; i < kPer; ++i) {
                const int c = threadIdx.x + i * kThreads;
                v[i] = c < d ? ld_cg(x + c) : 0.f;
                g[i] = c < d ? __ldg(gamma + c) : 0.f;
                b[i] = c < d ? __ldg(beta + c) : 0.f;
            }
            if (add.count > 0) {
                add_addends<kPer>(add, row, d, threadIdx.x, kThreads, v);
                if (add.sum_out) {
#pragma unroll
                    for (int i = 0; i < kPer; ++i) {
                        const int c = threadIdx.x + i * kThreads;
                        if (c < d) add.sum_out[row * d + c] = v[i];
                    }
                }
            }
            float total = 0.f;
#pragma unroll
            for (int i = 0; i < kPer; ++i) total += v[i];
            trl.end(kTrNormLoad);
            trl.begin();
            const float mean = consumer_sum_fresh(total, scratch[0]) / (float)d;
            float centred = 0.f;
#pragma unroll
            for (int i = 0; i < kPer; ++i) {
                const int c = threadIdx.x + i * kThreads;
                const float dv = c < d ? v[i] - mean : 0.f;
                centred += dv * dv;
            }
            const float scale = rsqrtf(consumer_sum_fresh(centred, scratch[1]) / (float)d + 1e-5f);
            WT* out = xs + (size_t)rl * ldx;
#pragma unroll
            for (int i = 0; i < kPer; ++i) {
                const int c = threadIdx.x + i * kThreads;
                if (c < d) {
                    const float y = (v[i] - mean) * scale * g[i] + b[i];
                    store_split(out + c, lo, y);
                    if (hidden_out) hidden_out[(size_t)(r0 + rl) * d + c] = y;
                }
            }
            for (int c = d + threadIdx.x; c < ldx; c += kThreads) out[c] = out[c + lo] = Half16<WT>::from_float(0.f);
            trl.end(kTrNormRest);
        }
        return;
    }
    // More rows: one warp a row, the row in registers.
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int rl = warp; rl < rows_in_tile; rl += kWarps) {
        const size_t row = (size_t)(r0 + rl) * row_step + row_offset;
        const float* x = input + row * d;
        float v[kNormMaxPerLane];
#pragma unroll
        for (int i = 0; i < kNormMaxPerLane; ++i) {
            const int c = lane + 32 * i;
            v[i] = c < d ? ld_cg(x + c) : 0.f;
        }
        if (add.count > 0) {
            add_addends<kNormMaxPerLane>(add, row, d, lane, 32, v);
            if (add.sum_out) {
#pragma unroll
                for (int i = 0; i < kNormMaxPerLane; ++i) {
                    const int c = lane + 32 * i;
                    if (c < d) add.sum_out[row * d + c] = v[i];
                }
            }
        }
        float total = 0.f;
#pragma unroll
        for (int i = 0; i < kNormMaxPerLane; ++i) total += v[i];
        const float mean = warp_sum(total) / (float)d;
        float centred = 0.f;
#pragma unroll
        for (int i = 0; i < kNormMaxPerLane; ++i) {
            const int c = lane + 32 * i;
            const float dv = c < d ? v[i] - mean : 0.f;
            centred += dv * dv;
        }
        const float scale = rsqrtf(warp_sum(centred) / (float)d + 1e-5f);
        // The gains and offsets are loaded in a loop with no stores, so they
        // can all be in flight together; the stores follow.
#pragma unroll
        for (int i = 0; i < kNormMaxPerLane; ++i) {
            const int c = lane + 32 * i;
            if (c < d) v[i] = (v[i] - mean) * scale * __ldg(gamma + c) + __ldg(beta + c);
        }
        WT* out = xs + (size_t)rl * ldx;
#pragma unroll
        for (int i = 0; i < kNormMaxPerLane; ++i) {
            const int c = lane + 32 * i;
            if (c < d) {
                store_split(out + c, lo, v[i]);
                if (hidden_out) hidden_out[(size_t)(r0 + rl) * d + c] = v[i];
            } else if (c < ldx) {
                out[c] = out[c + lo] = Half16<WT>::from_float(0.f);
            }
        }
    }
}

__device__ __forceinline__ int round16(int n) { return (n + 15) / 16 * 16; }

// Copies rows r0 .. r0+rows-1 of 16-bit rows X [.., ld] and of their lo
// plane (x_lo elements on) into the tile xs [rows][ldx] and xs + xs_lo, kp
// values a row (a multiple of 8), all loads in flight.
template <typename WT>
__device__ void stage_rows(const WT* X, int ld, size_t x_lo, int r0, int rows, int kp, WT* xs, int ldx,
                           size_t xs_lo) {
    const int per_row = kp / 8;
    const int total = rows * per_row;
#pragma unroll 4
    for (int i = threadIdx.x; i < total; i += kThreads) {
        const int rl = i / per_row, c = (i % per_row) * 8;
        const WT* from = X + (size_t)(r0 + rl) * ld + c;
        const uint4 hi = ld_cg4(from), lo = ld_cg4(from + x_lo);
        *reinterpret_cast<uint4*>(xs + (size_t)rl * ldx + c) = hi;
        *reinterpret_cast<uint4*>(xs + (size_t)rl * ldx + c + xs_lo) = lo;
    }
}

// LayerNorm of op.norm_rows rows into 16-bit rows (both planes), a row per
// CTA at a time with the whole CTA on it.
template <typename WT>
__device__ void op_norm(const StepParams& p, const StepOp& op, unsigned char* work) {
    WT* out = static_cast<WT*>(op.out);
    const size_t lo = lo_plane(p, op.ld_out);
    WT* row16 = reinterpret_cast<WT*>(work);  // the block layout: a row (hi, lo) first, then its pieces
    Addends add;
    if (op.addend_count > 0)
        add = Addends{op.addends, op.addend_count, op.addend_stride, op.addend_bias, op.sum_out, op.addend_tile_rows};
    for (int row = blockIdx.x; row < op.norm_rows; row += gridDim.x) {
        consumer_sync();
        if (!op.norm_umma) {
            layer_norm_tile<WT>(p, p.h, op.gamma, op.beta, row, 1, op.norm_step, op.norm_offset,
                                out + (size_t)row * op.ld_out, op.ld_out, lo, op.norm_hidden, add);
            continue;
        }
        layer_norm_tile<WT>(p, p.h, op.gamma, op.beta, row, 1, op.norm_step, op.norm_offset, row16, op.ld_out,
                            (size_t)op.ld_out, op.norm_hidden, add);
        consumer_sync();
        for (int c = 8 * threadIdx.x; c < op.ld_out; c += 8 * kThreads) {
            WT* at = out + act_offset(row, c, p.act_rows);
            *reinterpret_cast<uint4*>(at) = *reinterpret_cast<const uint4*>(row16 + c);
            *reinterpret_cast<uint4*>(at + lo) = *reinterpret_cast<const uint4*>(row16 + op.ld_out + c);
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
__device__ __forceinline__ void product_chunk(const unsigned char* unit, int c, const WT* X, int ldx, size_t x_lo,
                                              int k0, const bool (&x_ok)[NT], float (&acc)[NT][4]) {
    const int lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;
    const unsigned char* w = unit + (size_t)c * 1024 + lane * 16;
    const uint4 lo = *reinterpret_cast<const uint4*>(w), hi = *reinterpret_cast<const uint4*>(w + 512);
    uint4 B[NT], L[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const WT* at = X + (size_t)(x_ok[j] ? 8 * j + gq : 0) * ldx + k0 + 8 * tq;
        if (!x_ok[j]) {
            B[j] = L[j] = make_uint4(0, 0, 0, 0);
        } else if constexpr (X_SHARED) {
            B[j] = *reinterpret_cast<const uint4*>(at);
            L[j] = *reinterpret_cast<const uint4*>(at + x_lo);
        } else {
            B[j] = ld_cg4(at);
            L[j] = ld_cg4(at + x_lo);
        }
    }
    const uint32_t a0[4] = {lo.x, hi.x, lo.y, hi.y};
    const uint32_t a1[4] = {lo.z, hi.z, lo.w, hi.w};
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const uint32_t b0[2] = {B[j].x, B[j].y}, b1[2] = {B[j].z, B[j].w};
        const uint32_t l0[2] = {L[j].x, L[j].y}, l1[2] = {L[j].z, L[j].w};
        mma_16816<WT>(acc[j], a0, b0);
        mma_16816<WT>(acc[j], a1, b1);
        mma_16816<WT>(acc[j], a0, l0);
        mma_16816<WT>(acc[j], a1, l1);
    }
}

// Two chunks, c and c2, against the input rows: all fragments of both are
// loaded before the first MMA, and the products go to two independent sums
// (the k-halves alternate), so the warp waits on one MMA latency, not four.
template <typename WT, int NT, bool X_SHARED>
__device__ __forceinline__ void product_chunk_pair(const unsigned char* unit, int c, int c2, const WT* X, int ldx,
                                                   size_t x_lo, int k0, int k02, const bool (&x_ok)[NT],
                                                   float (&acc)[NT][4], float (&acc2)[NT][4]) {
    const int lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;
    const unsigned char* w = unit + (size_t)c * 1024 + lane * 16;
    const unsigned char* w2 = unit + (size_t)c2 * 1024 + lane * 16;
    const uint4 lo = *reinterpret_cast<const uint4*>(w), hi = *reinterpret_cast<const uint4*>(w + 512);
    const uint4 lo2 = *reinterpret_cast<const uint4*>(w2), hi2 = *reinterpret_cast<const uint4*>(w2 + 512);
    uint4 B[NT], B2[NT], L[NT], L2[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const WT* row = X + (size_t)(x_ok[j] ? 8 * j + gq : 0) * ldx + 8 * tq;
        if (!x_ok[j]) {
            B[j] = B2[j] = L[j] = L2[j] = make_uint4(0, 0, 0, 0);
        } else if constexpr (X_SHARED) {
            B[j] = *reinterpret_cast<const uint4*>(row + k0);
            B2[j] = *reinterpret_cast<const uint4*>(row + k02);
            L[j] = *reinterpret_cast<const uint4*>(row + x_lo + k0);
            L2[j] = *reinterpret_cast<const uint4*>(row + x_lo + k02);
        } else {
            B[j] = ld_cg4(row + k0);
            B2[j] = ld_cg4(row + k02);
            L[j] = ld_cg4(row + x_lo + k0);
            L2[j] = ld_cg4(row + x_lo + k02);
        }
    }
    const uint32_t a0[4] = {lo.x, hi.x, lo.y, hi.y}, a1[4] = {lo.z, hi.z, lo.w, hi.w};
    const uint32_t c0[4] = {lo2.x, hi2.x, lo2.y, hi2.y}, c1[4] = {lo2.z, hi2.z, lo2.w, hi2.w};
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const uint32_t b0[2] = {B[j].x, B[j].y}, b1[2] = {B[j].z, B[j].w};
        const uint32_t d0[2] = {B2[j].x, B2[j].y}, d1[2] = {B2[j].z, B2[j].w};
        const uint32_t l0[2] = {L[j].x, L[j].y}, l1[2] = {L[j].z, L[j].w};
        const uint32_t m0[2] = {L2[j].x, L2[j].y}, m1[2] = {L2[j].z, L2[j].w};
        mma_16816<WT>(acc[j], a0, b0);
        mma_16816<WT>(acc2[j], a1, b1);
        mma_16816<WT>(acc[j], c0, d0);
        mma_16816<WT>(acc2[j], c1, d1);
        mma_16816<WT>(acc[j], a0, l0);
        mma_16816<WT>(acc2[j], a1, l1);
        mma_16816<WT>(acc[j], c0, m0);
        mma_16816<WT>(acc2[j], c1, m1);
    }
}

// The warp's chunks c_first, c_first + step, ... (< n) of a unit, k offset
// k_base + 32 c, two at a time.
template <typename WT, int NT, bool X_SHARED>
__device__ __forceinline__ void chunks_product(const unsigned char* unit, int c_first, int step, int n, const WT* X,
                                               int ldx, size_t x_lo, int k_base, const bool (&x_ok)[NT],
                                               float (&acc)[NT][4]) {
    float acc2[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc2[j][0] = acc2[j][1] = acc2[j][2] = acc2[j][3] = 0.f;
    int c = c_first;
    for (; c + step < n; c += 2 * step)
        product_chunk_pair<WT, NT, X_SHARED>(unit, c, c + step, X, ldx, x_lo, k_base + c * 32,
                                             k_base + (c + step) * 32, x_ok, acc, acc2);
    if (c < n) product_chunk<WT, NT, X_SHARED>(unit, c, X, ldx, x_lo, k_base + c * 32, x_ok, acc2);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        acc[j][0] += acc2[j][0];
        acc[j][1] += acc2[j][1];
        acc[j][2] += acc2[j][2];
        acc[j][3] += acc2[j][3];
    }
}

// One 16-row tile over all of K: its units come off the weight stream in
// order, the 8 warps taking alternate chunks of each.  False if a wait gave
// up (the abort word is then raised and the kernel is on its way out).
template <typename WT, int NT, bool X_SHARED>
__device__ bool product_tile(const StepParams& p, Stream& s, int kp, const WT* X, int ldx, size_t x_lo,
                             int rows_valid, float (&acc)[NT][4]) {
    const int warp = threadIdx.x >> 5, gq = (threadIdx.x & 31) >> 2;
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    bool x_ok[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) x_ok[j] = 8 * j + gq < rows_valid;
    const int chunks = kp / 32;
    const int stage_chunks = s.stage_bytes / 1024;
    for (int c0 = 0; c0 < chunks; c0 += stage_chunks) {
        const int n = min(stage_chunks, chunks - c0);
        const unsigned char* unit = acquire_unit(p, s);
        if (!unit) return false;
        Trace tr = trace_of(p.profile);
        tr.begin();
        chunks_product<WT, NT, X_SHARED>(unit, warp, kWarps, n, X, ldx, x_lo, c0 * 32, x_ok, acc);
        tr.end(kTrCompute);
        release_unit(s);
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
    consumer_sync();
}

__device__ __forceinline__ float product_sum(const float* red, int RT, int nl, int rl) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[(w * 16 + nl) * RT + rl];
    return v;
}

// One output of a product, v = the row of x times weight row n plus the
// bias, written the way op.epilogue says (row r, at position + t of its
// window for the self caches).
template <typename WT>
__device__ __forceinline__ void emit_output(const StepParams& p, const StepOp& op, int position, int n, int r, float v) {
    switch (op.epilogue) {
    case kEpStore: {
        // Rows grouped by head, each head's rows padded to a whole tile.
        int col = n;
        if (op.slice > 0) {
            const int within = n % round16(op.slice);
            if (within >= op.slice) return;
            col = (n / round16(op.slice)) * op.slice + within;
        }
        static_cast<float*>(op.out)[(size_t)r * op.ld_out + col] = v;
        return;
    }
    case kEpResidual:
        // The one writer of this element in the op: a reduction
        // adds exactly what a read-add-write would, without waiting.
        atomicAdd(static_cast<float*>(op.out) + (size_t)r * op.ld_out + n, v);
        return;
    case kEpGelu:
        store_split(static_cast<WT*>(op.out) + act_index(p, r, n, op.ld_out), lo_plane(p, op.ld_out), gelu_exact(v));
        return;
    case kEpQkv: {
        // Head h's rows: its q, k and v rows, padded to a whole tile.
        const int D = p.head_width, group = round16(3 * D);
        const int within = n % group;
        if (within >= 3 * D) return;
        const int col = (n / group) * D + within % D;
        const int which = within / D;
        if (which == 0) {
            static_cast<float*>(op.out)[(size_t)r * op.ld_out + col] = v;
        } else {
            const int b = r / p.tokens, t = r % p.tokens;
            WT* cache = static_cast<WT*>(which == 1 ? op.self_keys : op.self_values);
            cache[((size_t)b * p.max_positions + position + t) * p.width + col] = Half16<WT>::from_float(v);
        }
        return;
    }
    }
}

// Work area of a product: [xs: 2 planes x RT x pitch 16-bit][red: 8 x 16 x RT][tile: 16 x RT]
//                         [best values: out_rows][best indices: out_rows]
template <typename WT, int NT>
__device__ void op_product(const StepParams& p, const StepOp& op, int position, Stream& s, unsigned char* work) {
    constexpr int RT = 8 * NT;
    const int pitch = tile_pitch(p.kpd);
    WT* xs = reinterpret_cast<WT*>(work);
    const size_t xs_lo = (size_t)RT * pitch;
    float* red = reinterpret_cast<float*>(work + 2 * xs_lo * sizeof(WT));
    const bool normalise = op.gamma != nullptr;
    const int n_tiles = (op.n + 15) / 16;
    const int r_tiles = (p.rows + RT - 1) / RT;
    // A split product (kEpPartial): kparts items a tile, each over its share
    // of K, reading its 16-bit input rows straight from memory.
    const int parts = op.kparts > 1 ? op.kparts : 1;
    const int kps = op.kp / parts;
    int cached_tile = -1;

    for (int item = blockIdx.x; item < n_tiles * r_tiles * parts; item += gridDim.x) {
        const int part = item / (n_tiles * r_tiles), rest = item % (n_tiles * r_tiles);
        const int r_tile = rest / n_tiles, n_tile = rest % n_tiles;
        const int r0 = r_tile * RT, n0 = n_tile * 16;
        const int rows_valid = min(RT, p.rows - r0);
        // This thread's outputs' biases, loaded now so the epilogue does not
        // wait on memory for them.  (A part's sums go out without it: the
        // op that adds the parts adds the bias.)
        constexpr int kOuts = (16 * RT + kThreads - 1) / kThreads;
        float bias_of[kOuts];
#pragma unroll
        for (int k = 0; k < kOuts; ++k) {
            const int n = n0 + (threadIdx.x + k * kThreads) / RT;
            bias_of[k] = op.bias && op.epilogue != kEpPartial && threadIdx.x + k * kThreads < 16 * RT && n < op.n
                             ? __ldg(op.bias + n)
                             : 0.f;
        }
        float acc[NT][4];
        bool ok;
        if (normalise || op.kp == p.kpd) {
            // The tile's input rows in shared memory, once per row tile:
            // normalised here, or copied from 16-bit rows.
            if (cached_tile != r_tile) {
                consumer_sync();
                Trace trn = trace_of(p.profile);
                trn.begin();
                if (normalise) {
                    // The residual additions of a fused out-projection; the
                    // CTA holding the row tile's first weight tile keeps them.
                    Addends add;
                    if (op.addend_count > 0) {
                        add = Addends{op.addends, op.addend_count, op.addend_stride, op.addend_bias,
                                      blockIdx.x == (unsigned)((r_tile * n_tiles) % gridDim.x) ? op.sum_out : nullptr};
                    }
                    layer_norm_tile<WT>(p, op.norm_input ? op.norm_input : p.h, op.gamma, op.beta, r0, rows_valid,
                                        1, 0, xs, pitch, xs_lo, nullptr, add);
                }
                else
                    stage_rows<WT>(static_cast<const WT*>(op.input16), op.ld_input, lo_plane(p, op.ld_input), r0,
                                   rows_valid, op.kp, xs, pitch, xs_lo);
                consumer_sync();
                trn.end(kTrNorm);
                cached_tile = r_tile;
            }
            ok = product_tile<WT, NT, true>(p, s, op.kp, xs, pitch, xs_lo, rows_valid, acc);
        } else {
            const WT* X = static_cast<const WT*>(op.input16) + (size_t)r0 * op.ld_input + (size_t)part * kps;
            ok = product_tile<WT, NT, false>(p, s, kps, X, op.ld_input, lo_plane(p, op.ld_input), rows_valid, acc);
        }
        if (!ok) return;
        Trace tre = trace_of(p.profile);
        tre.begin();
        product_reduce<NT>(red, acc);
#pragma unroll
        for (int k = 0; k < kOuts; ++k) {
            const int o = threadIdx.x + k * kThreads;
            if (o >= 16 * RT) break;
            const int nl = o / RT, rl = o % RT;
            const int n = n0 + nl, r = r0 + rl;
            if (n >= op.n || rl >= rows_valid) continue;
            if (op.epilogue == kEpPartial) {
                static_cast<float*>(op.out)[((size_t)part * p.rows + r) * op.ld_out + n] = product_sum(red, RT, nl, rl);
                continue;
            }
            emit_output<WT>(p, op, position, n, r, product_sum(red, RT, nl, rl) + bias_of[k]);
        }
        consumer_sync();
        tre.end(kTrEpilogue);
    }
}

// ------------------------------------------------------- tcgen05 products

// With many rows a product runs on the 5th-generation tensor cores: item
// (128 weight rows, up to umma_rows rows) accumulates D[128 x N] in tensor
// memory over the k-blocks of its weight tile and of the rows' activations,
// both streamed through the ring in the 128-byte-swizzled K-major layout
// (umma_offset / act_offset).  Lane 0 of warp kIssueWarp issues tcgen05.mma
// (M = 128, N = the rows rounded to 16, K = 16 per instruction, four per
// k-block); warps 0..3, whole warps since tcgen05.ld is warp-collective,
// read D back (lane = weight row) for the epilogue.
struct TensorMemory {
    uint32_t base;           // allocated columns (kTmemColumns), lanes 0..127
    uint64_t* done;          // the item's products completed (tcgen05.commit)
    uint32_t phase;
    // The activations' own ring in the work area: blocks of the rows an op
    // reads, fetched once the op has started (the weights' ring runs ahead
    // across ops).
    unsigned char* x_ring;
    uint64_t* x_full;        // [x_stages] the block landed
    uint64_t* x_empty;       // [x_stages] the products that read it completed
    int x_stages, x_stage_bytes;
    unsigned long long x_next;
    RingDivisor x_div;       // stage and round of an activation block
};
constexpr uint32_t kTmemColumns = 256;
constexpr int kLoadWarp = 5;      // lane 0 fetches the activation blocks
constexpr int kMaxXStages = 4;
constexpr int kIssueWarp = 4;  // not one of the epilogue warps 0..3
constexpr int kJoinLoads = 16;  // split partials a thread loads before summing

__device__ __forceinline__ void stage_arrive(const Stream& s, unsigned long long index, unsigned count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_address(s.empty + s.div.slot(index))),
                 "r"(count)
                 : "memory");
}
template <typename WT>
__device__ void product_umma(const StepParams& p, const StepOp& op, int position, int step, int op_index, Stream& s,
                             TensorMemory& tm) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tiles = (op.n + 127) / 128, groups = (p.rows + p.umma_rows - 1) / p.umma_rows;
    const int ks = op.ksplit > 1 ? op.ksplit : 1;
    const int items = m_tiles * groups * ks;
    const int row_stride = groups * p.umma_rows;  // of the partials
    __shared__ int join_ok;
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const UmmaItem u = umma_item(p, op, item);
        const int m = u.m, r0 = u.r0, rows = u.rows;
        const int nkb = u.kb1 - u.kb0;
        const int n16 = (rows + 15) & ~15;
        const unsigned long long x0 = tm.x_next;
        if (threadIdx.x == 32 * kLoadWarp) {
            // The rows' activation blocks, written by the ops before this one
            // (whose grid barrier has passed): generic writes ordered before
            // these bulk reads, then one copy a block into the X stages.
            asm volatile("fence.proxy.async.global;\n" ::: "memory");
            // Each stage takes the block's hi rows, then its lo rows (the lo
            // plane, act_rows * kp elements on).
            const unsigned char* src = static_cast<const unsigned char*>(op.input16) +
                                       ((size_t)u.kb0 * p.act_rows + r0) * 128;
            const size_t lo_bytes = lo_plane(p, op.kp) * 2;
            const unsigned bytes = (unsigned)n16 * 128u;
            for (int j = 0; j < nkb; ++j) {
                const unsigned long long q = x0 + j;
                const int st = (int)tm.x_div.slot(q);
                if (q >= (unsigned long long)tm.x_stages &&
                    !wait_parity(p, tm.x_empty + st, (tm.x_div.round(q) - 1u) & 1u, nullptr, kWaitEmpty, q))
                    break;
                const uint32_t bar = smem_address(tm.x_full + st);
                const uint32_t dst = smem_address(tm.x_ring + (size_t)st * tm.x_stage_bytes);
                const unsigned char* from = src + (size_t)j * p.act_rows * 128;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(2 * bytes)
                             : "memory");
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
                    "l"(from), "r"(bytes), "r"(bar)
                    : "memory");
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                        dst + bytes),
                    "l"(from + lo_bytes), "r"(bytes), "r"(bar)
                    : "memory");
            }
        }
        if (threadIdx.x == 32 * kIssueWarp) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t idesc = umma_idesc<WT>(n16);
            for (int j0 = 0; j0 < nkb; j0 += p.umma_blocks) {
                const unsigned long long iw = s.next + j0 / p.umma_blocks;
                const uint32_t w = smem_address(unit_at(p, s, iw));
                for (int j = j0; j < nkb && j < j0 + p.umma_blocks; ++j) {
                    const unsigned long long q = x0 + j;
                    const int st = (int)tm.x_div.slot(q);
                    wait_parity(p, tm.x_full + st, tm.x_div.round(q) & 1u, nullptr, kWaitUnit, q);
                    const uint32_t x = smem_address(tm.x_ring + (size_t)st * tm.x_stage_bytes);
                    const uint32_t x_lo = x + (uint32_t)n16 * 128u;
                    const uint32_t wb = w + (uint32_t)(j - j0) * 16384u;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        umma_mma(tm.base, umma_desc(wb + 32 * kk), umma_desc(x + 32 * kk), idesc, (j | kk) != 0);
                        umma_mma(tm.base, umma_desc(wb + 32 * kk), umma_desc(x_lo + 32 * kk), idesc, 1u);
                    }
                    umma_commit(tm.x_empty + st);  // the X stage: free once these products have read it
                }
                // The weight stage is free after kWarps arrivals: kWarps - 1
                // now, the last once the products above have read it.
                stage_arrive(s, iw, kWarps - 1);
                umma_commit(s.empty + s.div.slot(iw));
            }
            umma_commit(tm.done);
        }
        s.next += (unsigned long long)((nkb + p.umma_blocks - 1) / p.umma_blocks);
        tm.x_next += (unsigned long long)nkb;
        // Partials are [split][weight tile][row][128 weight rows]: an item's
        // block is contiguous, and a warp's lanes (consecutive weight rows)
        // store one row's 128 bytes at a time.  (Rows of the whole width
        // apart -- a power of two of bytes for every Whisper width -- the
        // stores crowded a few L2 slices.)
        const size_t split_stride = (size_t)m_tiles * row_stride * 128;
        float* partial = ks > 1 ? p.partial_d + (size_t)u.split * split_stride + ((size_t)m * row_stride + r0) * 128
                                : nullptr;
        if (warp < 4) {
            Trace tr = trace_of(p.profile);
            tr.begin();
            // (The bias loads while the products finish.)
            const int n = m * 128 + 32 * warp + lane;
            const float bias = op.bias && n < op.n ? __ldg(op.bias + n) : 0.f;
            wait_parity(p, tm.done, tm.phase, nullptr, kWaitUnit, (unsigned long long)item);
            __syncwarp();
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            for (int c0 = 0; c0 < n16; c0 += 32) {
                uint32_t v[32];
                tmem_load32(tm.base + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, v);
                if (partial) {
                    float* col = partial + (size_t)c0 * 128 + 32 * warp + lane;
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (c0 + j < rows) col[j * 128] = __uint_as_float(v[j]);
                } else if (n < op.n) {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (c0 + j < rows) emit_output<WT>(p, op, position, n, r0 + c0 + j, __uint_as_float(v[j]) + bias);
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            tr.end(kTrEpilogue);
        }
        tm.phase ^= 1u;
        if (ks > 1 && !op.defer_join) {
            // The tile's splits (each on its own CTA: a split product's items
            // fit one wave) meet here; then each joins a contiguous share of
            // the tile's (row, weight row) elements, summing the partials in
            // split order.  (The release below, after the CTA barrier,
            // publishes every thread's partials.)
            consumer_sync();
            if (threadIdx.x == 0) {
                unsigned* counter = p.split_counters + (size_t)op_index * kSplitSlots + (item % (m_tiles * groups));
                asm volatile("red.release.gpu.global.add.u32 [%0], %1;\n" ::"l"(counter), "r"(1u) : "memory");
                const unsigned target = (unsigned)(step + 1) * (unsigned)ks;
                const unsigned long long start = global_ns();
                int ok = 1;
                for (unsigned spin = 1; ld_acquire(counter) < target; ++spin) {
                    if ((spin & 15) != 0) continue;
                    if (ld_volatile(p.state + kAbort)) { ok = 0; break; }
                    if (global_ns() - start > kWaitTimeoutNs) {
                        record_timeout(p, kWaitJoin, (long long)item);
                        ok = 0;
                        break;
                    }
                }
                join_ok = ok;
            }
            consumer_sync();
            if (join_ok) {
                // Four adjacent weight rows a thread.  Every split's partials
                // of them and their biases are loaded before any sum (up to
                // kJoinLoads splits at once: one round trip to L2 for 16
                // splits or fewer) and summed in split order.
                const int elems = rows * 128;
                const int per = ((elems + ks - 1) / ks + 3) & ~3;
                const int f1 = min((u.split + 1) * per, elems);
                const float* tile = p.partial_d + ((size_t)m * row_stride + r0) * 128;
                for (int f = u.split * per + 4 * threadIdx.x; f < f1; f += 4 * kThreads) {
                    const int t = f >> 7, nl = f & 127;
                    float b[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int n = m * 128 + nl + e;
                        b[e] = op.bias && n < op.n ? __ldg(op.bias + n) : 0.f;
                    }
                    float sum[4] = {0.f, 0.f, 0.f, 0.f};
                    for (int k0 = 0; k0 < ks; k0 += kJoinLoads) {
                        float4 v[kJoinLoads];
#pragma unroll
                        for (int k = 0; k < kJoinLoads; ++k)
                            v[k] = k0 + k < ks
                                       ? __ldcg(reinterpret_cast<const float4*>(tile + (k0 + k) * split_stride + f))
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (int k = 0; k < kJoinLoads; ++k)
                            if (k0 + k < ks) {
                                sum[0] += v[k].x;
                                sum[1] += v[k].y;
                                sum[2] += v[k].z;
                                sum[3] += v[k].w;
                            }
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int n = m * 128 + nl + e;
                        if (n < op.n) emit_output<WT>(p, op, position, n, r0 + t, sum[e] + b[e]);
                    }
                }
            }
        }
        consumer_sync();
    }
}

// ------------------------------------------------------------------- logits

// This CTA's per-row candidates best_v/best_i (shared memory, out_rows
// each), then the fold of every CTA's by whichever CTA finishes last: it
// writes each window's sampled id into its next token slot and advances the
// position (Argmax.h:83-201's two passes, across CTAs).
__device__ void logits_fold(const StepParams& p, int position, const float* best_v, const uint32_t* best_i) {
    __shared__ int is_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // This CTA's candidates, then the fold by whichever CTA finishes last.
    Trace trf = trace_of(p.profile);
    trf.begin();
    for (int r = threadIdx.x; r < p.out_rows; r += kThreads) {
        p.candidate_values[(size_t)r * gridDim.x + blockIdx.x] = best_v[r];
        p.candidate_indices[(size_t)r * gridDim.x + blockIdx.x] = best_i[r];
    }
    consumer_sync();
    if (threadIdx.x == 0) is_last = arrive_acq_rel(p.logits_counter) == gridDim.x - 1;
    consumer_sync();
    if (!is_last) {
        trf.end(kTrLogitsFold);
        return;
    }
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
    consumer_sync();
    if (threadIdx.x == 0) {
        if (p.stop_enabled) {
            int all = 1;
            for (int b = 0; b < p.windows; ++b) all &= p.ended[b] ? 1 : 0;
            if (all) atomicExch(p.state + kAllEnded, 1);
        }
        atomicAdd(p.state + kStepsDone, 1);
        atomicAdd(p.state + kPosition, p.tokens);
        atomicExch(p.logits_counter, 0u);
        // (The grid barrier after this op releases these writes.)
    }
    trf.end(kTrLogitsFold);
}

// LN(h) of the sampled rows against the tied token table, with the masked
// argmax folded in: each CTA keeps, per row, the first maximum over the
// columns it produced; the last CTA to finish folds the CTAs' candidates,
// writes each window's sampled id into its next token slot and advances the
// position.
template <typename WT, int NT>
__device__ void op_logits(const StepParams& p, const StepOp& op, int position, Stream& s, unsigned char* work) {
    constexpr int RT = 8 * NT;
    const int pitch = tile_pitch(p.kpd);
    WT* xs = reinterpret_cast<WT*>(work);
    const size_t xs_lo = (size_t)RT * pitch;
    float* fold_v = reinterpret_cast<float*>(work + 2 * xs_lo * sizeof(WT));  // [8 warps][RT]
    uint32_t* fold_i = reinterpret_cast<uint32_t*>(fold_v + kWarps * RT);
    float* best_v = reinterpret_cast<float*>(fold_i + kWarps * RT);
    uint32_t* best_i = reinterpret_cast<uint32_t*>(best_v + p.out_rows);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;

    for (int r = threadIdx.x; r < p.out_rows; r += kThreads) {
        best_v[r] = -INFINITY;
        best_i[r] = kUnchosen;
    }
    const int n_tiles = (p.vocabulary + 15) / 16;
    const int r_tiles = (p.out_rows + RT - 1) / RT;
    const int chunks = p.kpd / 32;
    const int stage_chunks = s.stage_bytes / 1024;
    const int blocks = (chunks + stage_chunks - 1) / stage_chunks;  // units of a tile
    const unsigned long long base = s.next;
    int mine = 0;  // this CTA's items so far (unit index = base + mine*blocks + block)

    // A row tile at a time: the CTA normalises its rows, then every warp
    // takes whole vocabulary tiles of it -- tile k of the CTA goes to warp
    // k % 8 -- over all of K, keeping per row the first maximum it meets.
    for (int r_tile = 0; r_tile < r_tiles; ++r_tile) {
        const int lo = r_tile * n_tiles, hi = lo + n_tiles;
        int first = blockIdx.x;
        if (first < lo) first += ((lo - first + gridDim.x - 1) / gridDim.x) * gridDim.x;
        if (first >= hi) continue;
        const int count = (hi - first + gridDim.x - 1) / gridDim.x;
        const int r0 = r_tile * RT;
        const int rows_valid = min(RT, p.out_rows - r0);
        consumer_sync();
        Trace trn = trace_of(p.profile);
        trn.begin();
        if (op.input16)  // rows normalised by a norm op
            stage_rows<WT>(static_cast<const WT*>(op.input16), op.ld_input, lo_plane(p, op.ld_input), r0, rows_valid,
                           p.kpd, xs, pitch, xs_lo);
        else
            layer_norm_tile<WT>(p, p.h, p.final_gamma, p.final_beta, r0, rows_valid, p.row_step, p.row_offset, xs,
                                pitch, xs_lo, p.hidden_out);
        consumer_sync();
        trn.end(kTrNorm);

        Trace trt = trace_of(p.profile);
        trt.begin();
        bool x_ok[NT];
#pragma unroll
        for (int j = 0; j < NT; ++j) x_ok[j] = 8 * j + gq < rows_valid;
        float cand_v[NT][2];
        uint32_t cand_i[NT][2];
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            cand_v[j][0] = cand_v[j][1] = -INFINITY;
            cand_i[j][0] = cand_i[j][1] = kUnchosen;
        }
        for (int k = warp; k < count; k += kWarps) {
            const int n0 = (first - lo + k * (int)gridDim.x) * 16;
            // Lane (g, t) holds rows n0+g and n0+g+8 of input rows 8j+2t, 8j+2t+1;
            // their mask entries load now, under the tile's products.
            const int na = n0 + gq, nb = n0 + gq + 8;
            const bool a_ok = na < p.vocabulary && (p.mask == nullptr || __ldg(p.mask + na) == 0.f);
            const bool b_ok = nb < p.vocabulary && (p.mask == nullptr || __ldg(p.mask + nb) == 0.f);
            float acc[NT][4];
#pragma unroll
            for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
            for (int b = 0; b < blocks; ++b) {
                const unsigned long long index = base + (unsigned long long)(mine + k) * blocks + b;
                const unsigned char* unit = owned_unit_at(p, s, index);
                Trace tr = trace_of(p.profile);
                tr.begin();
                const int c0 = b * stage_chunks, n = min(stage_chunks, chunks - c0);
                chunks_product<WT, NT, true>(unit, 0, 1, n, xs, pitch, xs_lo, c0 * 32, x_ok, acc);
                tr.end(kTrCompute);
                release_at(s, index, kWarps);
            }
#pragma unroll
            for (int j = 0; j < NT; ++j) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int rl = 8 * j + 2 * tq + e;
                    if (rl >= rows_valid) continue;
                    const float va = acc[j][e], vb = acc[j][2 + e];
                    if (p.logits_out) {
                        if (na < p.vocabulary) p.logits_out[(size_t)(r0 + rl) * p.vocabulary + na] = va;
                        if (nb < p.vocabulary) p.logits_out[(size_t)(r0 + rl) * p.vocabulary + nb] = vb;
                    }
                    if (a_ok && candidate_better(va, (uint32_t)na, cand_v[j][e], cand_i[j][e])) {
                        cand_v[j][e] = va;
                        cand_i[j][e] = (uint32_t)na;
                    }
                    if (b_ok && candidate_better(vb, (uint32_t)nb, cand_v[j][e], cand_i[j][e])) {
                        cand_v[j][e] = vb;
                        cand_i[j][e] = (uint32_t)nb;
                    }
                }
            }
        }
        // Fold the warp's lanes of equal t (the 8 values of g), then the warps.
#pragma unroll
        for (int j = 0; j < NT; ++j) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                float bv = cand_v[j][e];
                uint32_t bi = cand_i[j][e];
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (candidate_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
                }
                if (gq == 0) {
                    fold_v[warp * RT + 8 * j + 2 * tq + e] = bv;
                    fold_i[warp * RT + 8 * j + 2 * tq + e] = bi;
                }
            }
        }
        consumer_sync();
        for (int rl = threadIdx.x; rl < rows_valid; rl += kThreads) {
            float bv = best_v[r0 + rl];
            uint32_t bi = best_i[r0 + rl];
            for (int w = 0; w < kWarps; ++w)
                if (candidate_better(fold_v[w * RT + rl], fold_i[w * RT + rl], bv, bi)) {
                    bv = fold_v[w * RT + rl];
                    bi = fold_i[w * RT + rl];
                }
            best_v[r0 + rl] = bv;
            best_i[r0 + rl] = bi;
        }
        mine += count;
        trt.end(kTrLogitsTiles);
    }
    s.next = base + (unsigned long long)mine * blocks;
    consumer_sync();

    logits_fold(p, position, best_v, best_i);
}

// With the tensor-core products the logits are tcgen05 tiles too (the
// token table is in their layout): item (128 vocabulary rows, up to 128
// sampled rows), the table's k-blocks off the weight ring, the rows'
// normalised hi and lo blocks off the activation ring, both products into
// one accumulator (lane = vocabulary row, column = sampled row).  Warps 0..3
// read it back 32 columns at a time into shared memory, [vocabulary row]
// [row], masked; then every consumer thread takes a share of one row's 128
// entries, ascending, and the shares fold in order into the CTA's per-row
// first maximum.  The fold across CTAs is logits_fold's.
// Work area: [activation ring | tile: 128 x 33, shares: 2 x kWarps x 32]
// [best values: out_rows][best indices: out_rows] -- the tile scratch
// shares the activation ring's bytes: a tile is read back only once every
// product of its item has completed, and the next item's blocks are fetched
// after the CTA barrier that ends the item.
constexpr int kLogitsTilePitch = 33;
constexpr int kLogitsScratchBytes = (int)sizeof(float) * (128 * kLogitsTilePitch + 2 * kWarps * 32);

template <typename WT>
__device__ void logits_umma(const StepParams& p, const StepOp& op, int position, Stream& s, TensorMemory& tm) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t ring_bytes = (size_t)tm.x_stages * tm.x_stage_bytes;
    float* tile = reinterpret_cast<float*>(tm.x_ring);
    float* best_v = reinterpret_cast<float*>(tm.x_ring + max(ring_bytes, (size_t)kLogitsScratchBytes));
    uint32_t* best_i = reinterpret_cast<uint32_t*>(best_v + p.out_rows);
    float* share_v = tile + 128 * kLogitsTilePitch;
    uint32_t* share_i = reinterpret_cast<uint32_t*>(share_v + kWarps * 32);
    for (int r = threadIdx.x; r < p.out_rows; r += kThreads) {
        best_v[r] = -INFINITY;
        best_i[r] = kUnchosen;
    }
    const int vocab_tiles = (p.vocabulary + 127) / 128;
    const int row_tiles = (p.out_rows + 127) / 128;
    const int kblocks = p.kpd / 64;
    const size_t lo_bytes = lo_plane(p, op.ld_input) * 2;
    for (int item = blockIdx.x; item < vocab_tiles * row_tiles; item += gridDim.x) {
        const int m = item % vocab_tiles, r0 = (item / vocab_tiles) * 128;
        const int rows = min(128, p.out_rows - r0), n16 = (rows + 15) & ~15;
        const unsigned long long x0 = tm.x_next;
        if (threadIdx.x == 32 * kLoadWarp) {
            // The rows' normalised blocks (the norm op before this one wrote
            // them): hi, then lo, one stage a k-block.
            asm volatile("fence.proxy.async.global;\n" ::: "memory");
            const unsigned char* src = static_cast<const unsigned char*>(op.input16) + (size_t)r0 * 128;
            const unsigned bytes = (unsigned)n16 * 128u;
            for (int j = 0; j < kblocks; ++j) {
                const unsigned long long q = x0 + j;
                const int st = (int)tm.x_div.slot(q);
                if (q >= (unsigned long long)tm.x_stages &&
                    !wait_parity(p, tm.x_empty + st, (tm.x_div.round(q) - 1u) & 1u, nullptr, kWaitEmpty, q))
                    break;
                const uint32_t bar = smem_address(tm.x_full + st);
                const uint32_t dst = smem_address(tm.x_ring + (size_t)st * tm.x_stage_bytes);
                const unsigned char* from = src + (size_t)j * p.act_rows * 128;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(2 * bytes)
                             : "memory");
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
                    "l"(from), "r"(bytes), "r"(bar)
                    : "memory");
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                        dst + bytes),
                    "l"(from + lo_bytes), "r"(bytes), "r"(bar)
                    : "memory");
            }
        }
        if (threadIdx.x == 32 * kIssueWarp) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t idesc = umma_idesc<WT>(n16);
            for (int j0 = 0; j0 < kblocks; j0 += p.umma_blocks) {
                const unsigned long long iw = s.next + j0 / p.umma_blocks;
                const uint32_t w = smem_address(unit_at(p, s, iw));
                for (int j = j0; j < kblocks && j < j0 + p.umma_blocks; ++j) {
                    const unsigned long long q = x0 + j;
                    const int st = (int)tm.x_div.slot(q);
                    wait_parity(p, tm.x_full + st, tm.x_div.round(q) & 1u, nullptr, kWaitUnit, q);
                    const uint32_t x = smem_address(tm.x_ring + (size_t)st * tm.x_stage_bytes);
                    const uint32_t x_lo = x + (uint32_t)n16 * 128u;
                    const uint32_t wb = w + (uint32_t)(j - j0) * 16384u;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        umma_mma(tm.base, umma_desc(wb + 32 * kk), umma_desc(x + 32 * kk), idesc, (j | kk) != 0);
                        umma_mma(tm.base, umma_desc(wb + 32 * kk), umma_desc(x_lo + 32 * kk), idesc, 1u);
                    }
                    umma_commit(tm.x_empty + st);
                }
                stage_arrive(s, iw, kWarps - 1);
                umma_commit(s.empty + s.div.slot(iw));
            }
            umma_commit(tm.done);
        }
        s.next += (unsigned long long)((kblocks + p.umma_blocks - 1) / p.umma_blocks);
        tm.x_next += (unsigned long long)kblocks;
        // This thread's vocabulary row (warps 0..3) and whether it may win.
        const int n = m * 128 + 32 * warp + lane;
        const bool pick = warp < 4 && n < p.vocabulary && (p.mask == nullptr || __ldg(p.mask + n) == 0.f);
        if (warp < 4) {
            wait_parity(p, tm.done, tm.phase, nullptr, kWaitUnit, (unsigned long long)item);
            __syncwarp();
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        }
        tm.phase ^= 1u;
        for (int c0 = 0; c0 < n16; c0 += 32) {
            consumer_sync();  // the tile scratch is free
            if (warp < 4) {
                uint32_t v[32];
                tmem_load32(tm.base + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float value = __uint_as_float(v[j]);
                    if (p.logits_out && n < p.vocabulary && c0 + j < rows)
                        p.logits_out[(size_t)(r0 + c0 + j) * p.vocabulary + n] = value;
                    tile[(32 * warp + lane) * kLogitsTilePitch + j] = pick ? value : -INFINITY;
                }
            }
            consumer_sync();
            // Thread (part, column): vocabulary rows part*19 .. of column j.
            const int j = threadIdx.x & 31, part = threadIdx.x >> 5;
            float bv = -INFINITY;
            uint32_t bi = kUnchosen;
            for (int t = part * 19; t < min(128, part * 19 + 19); ++t) {
                const float value = tile[t * kLogitsTilePitch + j];
                const uint32_t index = (uint32_t)(m * 128 + t);
                if (value != -INFINITY && candidate_better(value, index, bv, bi)) {
                    bv = value;
                    bi = index;
                }
            }
            share_v[part * 32 + j] = bv;
            share_i[part * 32 + j] = bi;
            consumer_sync();
            if (threadIdx.x < 32 && c0 + threadIdx.x < rows) {
                const int r = r0 + c0 + threadIdx.x;
                float v0 = best_v[r];
                uint32_t i0 = best_i[r];
                for (int w = 0; w < kWarps; ++w)
                    if (candidate_better(share_v[w * 32 + threadIdx.x], share_i[w * 32 + threadIdx.x], v0, i0)) {
                        v0 = share_v[w * 32 + threadIdx.x];
                        i0 = share_i[w * 32 + threadIdx.x];
                    }
                best_v[r] = v0;
                best_i[r] = i0;
            }
        }
        if (warp < 4) asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        consumer_sync();
    }
    logits_fold(p, position, best_v, best_i);
}

// ------------------------------------------------ fused out-projection

// Head `head`'s share of the attention out-projection for row r: the d
// outputs W[:, 64 head .. 64 head + 63] . a, with a the head's 64 attended
// values (16-bit, shared memory, 16-byte aligned: hi a[0..63], lo
// a[64..127], both multiplied), written to op.out_partial
// [head][r][:] (Decoder.cpp:80-104 adds out_proj(attention) to h; the op
// after this one adds the heads' partials in head order, with the bias).
// The head's columns are chunks 2 head and 2 head + 1 of every 16-row tile
// of the fragment-packed weight, read straight from memory (which CTA joins
// a (row, head) is known only at run time, so they are not on the stream).
// The CTA takes the output tiles first, first + step, ... (all of them when
// one CTA projects the head; a share when several do); its warps take those
// in turn, six tiles' fragments in flight at once, a as the one input row of
// swap-AB m16n8k16 products.
template <typename WT>
__device__ void head_out_projection(const StepParams& p, const StepOp& op, int r, int head, const WT* a,
                                    int first = 0, int step = 1) {
    Trace tr = trace_of(p.profile);
    tr.begin();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
    const int d = p.width, chunks = p.kpd / 32;
    const int tiles = ((d + 15) / 16 - first + step - 1) / step;  // this CTA's
    const uint4 zero = make_uint4(0, 0, 0, 0);
    const uint4 x0 = gq == 0 ? *reinterpret_cast<const uint4*>(a + 8 * tq) : zero;
    const uint4 x1 = gq == 0 ? *reinterpret_cast<const uint4*>(a + 32 + 8 * tq) : zero;
    const uint4 y0 = gq == 0 ? *reinterpret_cast<const uint4*>(a + 64 + 8 * tq) : zero;
    const uint4 y1 = gq == 0 ? *reinterpret_cast<const uint4*>(a + 96 + 8 * tq) : zero;
    const unsigned char* wbase = static_cast<const unsigned char*>(op.out_weight);
    float* out = op.out_partial + ((size_t)head * p.rows + r) * d;
    constexpr int kBatch = 6;
    for (int t0 = warp; t0 < tiles; t0 += kWarps * kBatch) {
        uint4 w[kBatch][4];
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const int t = first + (t0 + i * kWarps) * step;
            if (t0 + i * kWarps < tiles) {
                const unsigned char* src = wbase + ((size_t)t * chunks + 2 * head) * 1024 + lane * 16;
                w[i][0] = ld_nc4(reinterpret_cast<const uint4*>(src));
                w[i][1] = ld_nc4(reinterpret_cast<const uint4*>(src + 512));
                w[i][2] = ld_nc4(reinterpret_cast<const uint4*>(src + 1024));  // the next chunk
                w[i][3] = ld_nc4(reinterpret_cast<const uint4*>(src + 1536));
            } else {
                w[i][0] = w[i][1] = w[i][2] = w[i][3] = zero;
            }
        }
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const int t = first + (t0 + i * kWarps) * step;
            if (t0 + i * kWarps >= tiles) break;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            const uint32_t a0[4] = {w[i][0].x, w[i][1].x, w[i][0].y, w[i][1].y};
            const uint32_t a1[4] = {w[i][0].z, w[i][1].z, w[i][0].w, w[i][1].w};
            const uint32_t a2[4] = {w[i][2].x, w[i][3].x, w[i][2].y, w[i][3].y};
            const uint32_t a3[4] = {w[i][2].z, w[i][3].z, w[i][2].w, w[i][3].w};
            const uint32_t b0[2] = {x0.x, x0.y}, b1[2] = {x0.z, x0.w};
            const uint32_t b2[2] = {x1.x, x1.y}, b3[2] = {x1.z, x1.w};
            const uint32_t c0[2] = {y0.x, y0.y}, c1[2] = {y0.z, y0.w};
            const uint32_t c2[2] = {y1.x, y1.y}, c3[2] = {y1.z, y1.w};
            mma_16816<WT>(acc, a0, b0);
            mma_16816<WT>(acc, a1, b1);
            mma_16816<WT>(acc, a2, b2);
            mma_16816<WT>(acc, a3, b3);
            mma_16816<WT>(acc, a0, c0);
            mma_16816<WT>(acc, a1, c1);
            mma_16816<WT>(acc, a2, c2);
            mma_16816<WT>(acc, a3, c3);
            // Column 0 (the one input row) sits in lanes tq == 0: weight rows gq, gq + 8.
            if (tq == 0) {
                const int n = 16 * t + gq;
                if (n < d) out[n] = acc[0];
                if (n + 8 < d) out[n + 8] = acc[2];
            }
        }
    }
    tr.end(kTrOutProj);
}

// ----------------------------------------------------------------- attention

template <typename WT, bool READ_ONLY>
__device__ __forceinline__ uint4 load_kv4(const WT* at) {
    return READ_ONLY ? ld_nc4(at) : ld_cg4(at);
}
template <typename WT, bool READ_ONLY>
__device__ __forceinline__ float load_kv1(const WT* at) {
    return bits_to_float<WT>(READ_ONLY ? ld_nc_u16(at) : ld_cg_u16(at));
}

// q . K[key] over a 64-wide head: the key row's eight 16-byte pieces are all
// loaded before any is used, so a score costs one memory latency.
template <typename WT, bool READ_ONLY>
__device__ __forceinline__ float score64(const float* q, const WT* krow) {
    uint4 u[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) u[i] = load_kv4<WT, READ_ONLY>(krow + 8 * i);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float2 f0 = Half16<WT>::pair_to_float2(u[i].x), f1 = Half16<WT>::pair_to_float2(u[i].y);
        const float2 f2 = Half16<WT>::pair_to_float2(u[i].z), f3 = Half16<WT>::pair_to_float2(u[i].w);
        const float* qq = q + 8 * i;
        s += qq[0] * f0.x + qq[1] * f0.y + qq[2] * f1.x + qq[3] * f1.y + qq[4] * f2.x + qq[5] * f2.y + qq[6] * f3.x +
             qq[7] * f3.y;
    }
    return s;
}

template <typename WT, bool READ_ONLY>
__device__ __forceinline__ float score_any(const float* q, const WT* krow, int D) {
    if (D == 64) return score64<WT, READ_ONLY>(q, krow);
    float s = 0.f;
    if (D % 8 == 0) {
        for (int c = 0; c < D; c += 8) {
            const uint4 u = load_kv4<WT, READ_ONLY>(krow + c);
            const float2 f0 = Half16<WT>::pair_to_float2(u.x), f1 = Half16<WT>::pair_to_float2(u.y);
            const float2 f2 = Half16<WT>::pair_to_float2(u.z), f3 = Half16<WT>::pair_to_float2(u.w);
            s += q[c] * f0.x + q[c + 1] * f0.y + q[c + 2] * f1.x + q[c + 3] * f1.y + q[c + 4] * f2.x +
                 q[c + 5] * f2.y + q[c + 6] * f3.x + q[c + 7] * f3.y;
        }
    } else {
        for (int c = 0; c < D; ++c) s += q[c] * load_kv1<WT, READ_ONLY>(krow + c);
    }
    return s;
}

// Scores of keys [k0, k0+n) against q (in shared, pre-scaled), into scores[],
// a thread per key; returns this thread's maximum.
template <typename WT, bool READ_ONLY>
__device__ __forceinline__ float attention_scores(const float* q, const WT* K, long long key_stride, int D, int k0,
                                                  int n, float* scores) {
    float local_max = -INFINITY;
    for (int j = threadIdx.x; j < n; j += kThreads) {
        const float s = score_any<WT, READ_ONLY>(q, K + (size_t)(k0 + j) * key_stride, D);
        scores[j] = s;
        local_max = fmaxf(local_max, s);
    }
    return local_max;
}

// sum_j p_j V[k0 + j] over the keys into result[0..D).  With D a multiple
// of 8, thread (group, piece) reads 16 bytes of a value row per key, four
// keys' loads in flight at a time, and the 256/(D/8) key groups fold in
// shared memory (fold holds 2048 floats).
template <typename WT, bool READ_ONLY>
__device__ __forceinline__ void attention_values(const float* scores, const WT* V, long long key_stride, int D,
                                                 int k0, int n, float* fold, float* result) {
    if (D % 8 == 0) {
        const int pieces = D / 8;
        const int groups = kThreads / pieces;
        const int piece = threadIdx.x % pieces, g = threadIdx.x / pieces;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (g < groups) {
#pragma unroll 8
            for (int j = g; j < n; j += groups) {
                const uint4 u = load_kv4<WT, READ_ONLY>(V + (size_t)(k0 + j) * key_stride + piece * 8);
                const float w = scores[j];
                const float2 f0 = Half16<WT>::pair_to_float2(u.x), f1 = Half16<WT>::pair_to_float2(u.y);
                const float2 f2 = Half16<WT>::pair_to_float2(u.z), f3 = Half16<WT>::pair_to_float2(u.w);
                acc[0] += w * f0.x; acc[1] += w * f0.y; acc[2] += w * f1.x; acc[3] += w * f1.y;
                acc[4] += w * f2.x; acc[5] += w * f2.y; acc[6] += w * f3.x; acc[7] += w * f3.y;
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) fold[g * D + piece * 8 + e] = acc[e];
        }
        consumer_sync();
        if (threadIdx.x < D) {
            float o = 0.f;
            for (int gg = 0; gg < groups; ++gg) o += fold[gg * D + threadIdx.x];
            result[threadIdx.x] = o;
        }
    } else {
        const int groups = kThreads / D;
        const int c = threadIdx.x % D, g = threadIdx.x / D;
        float acc = 0.f;
        if (g < groups) {
#pragma unroll 4
            for (int j = g; j < n; j += groups)
                acc += scores[j] * load_kv1<WT, READ_ONLY>(V + (size_t)(k0 + j) * key_stride + c);
            fold[g * D + c] = acc;
        }
        consumer_sync();
        if (threadIdx.x < D) {
            float o = 0.f;
            for (int gg = 0; gg < groups; ++gg) o += fold[gg * D + threadIdx.x];
            result[threadIdx.x] = o;
        }
    }
    consumer_sync();
}

// Shared memory of attention: [q: 64][scratch: 8][fold: 2048][result: 64][scores: ...]
constexpr int kFold = 2048;
constexpr int kAttentionFixed = 64 + 8 + kFold + 64;

// Self-attention of row (b, t) and head h over keys 0..position+t: one item.
// A self-attention item of at most kThreads keys and 64-wide heads: thread
// j loads key row j, and thread (g, piece) the value pieces of keys g, g +
// 28, ..., all before q arrives, so the item waits on memory once.  Scores
// (scaled q . k), the maximum, the weights exp(s - max) and their sum, and
// the weighted values as the general path computes them
// (SingleQueryAttention.h:62-373); returns the sum, result[0..63] holds the
// unnormalised output.
template <typename WT>
__device__ float self_item_in_registers(const StepParams& p, int r, int head, int keys, const WT* K, const WT* V,
                                        long long key_stride, float* q, float* scratch, float* fold, float* result,
                                        float* scores) {
    const int j = threadIdx.x;
    const uint4 zero = make_uint4(0, 0, 0, 0);
    uint4 kr[8], vr[8];
    const WT* krow = K + (size_t)(j < keys ? j : 0) * key_stride;
#pragma unroll
    for (int i = 0; i < 8; ++i) kr[i] = j < keys ? load_kv4<WT, false>(krow + 8 * i) : zero;
    constexpr int kGroups = kThreads / 8;
    const int piece = threadIdx.x & 7, g = threadIdx.x >> 3;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int key = g + kGroups * i;
        vr[i] = key < keys ? load_kv4<WT, false>(V + (size_t)key * key_stride + piece * 8) : zero;
    }
    if (threadIdx.x < 64) q[threadIdx.x] = ld_cg(p.q + (size_t)r * p.width + head * 64 + threadIdx.x) * p.scale;
    consumer_sync();
    float sc = -INFINITY;
    if (j < keys) {
        sc = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float2 f0 = Half16<WT>::pair_to_float2(kr[i].x), f1 = Half16<WT>::pair_to_float2(kr[i].y);
            const float2 f2 = Half16<WT>::pair_to_float2(kr[i].z), f3 = Half16<WT>::pair_to_float2(kr[i].w);
            const float* qq = q + 8 * i;
            sc += qq[0] * f0.x + qq[1] * f0.y + qq[2] * f1.x + qq[3] * f1.y + qq[4] * f2.x + qq[5] * f2.y +
                  qq[6] * f3.x + qq[7] * f3.y;
        }
    }
    const float m = consumer_max(sc, scratch);
    const float e = j < keys ? __expf(sc - m) : 0.f;
    if (j < keys) scores[j] = e;
    const float l = consumer_sum(e, scratch);  // (its barriers also publish scores[])
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int key = g + kGroups * i;
        if (key >= keys) break;
        const float w = scores[key];
        const float2 f0 = Half16<WT>::pair_to_float2(vr[i].x), f1 = Half16<WT>::pair_to_float2(vr[i].y);
        const float2 f2 = Half16<WT>::pair_to_float2(vr[i].z), f3 = Half16<WT>::pair_to_float2(vr[i].w);
        acc[0] += w * f0.x; acc[1] += w * f0.y; acc[2] += w * f1.x; acc[3] += w * f1.y;
        acc[4] += w * f2.x; acc[5] += w * f2.y; acc[6] += w * f3.x; acc[7] += w * f3.y;
    }
#pragma unroll
    for (int e8 = 0; e8 < 8; ++e8) fold[g * 64 + piece * 8 + e8] = acc[e8];
    consumer_sync();
    if (threadIdx.x < 64) {
        float o = 0.f;
        for (int gg = 0; gg < kGroups; ++gg) o += fold[gg * 64 + threadIdx.x];
        result[threadIdx.x] = o;
    }
    consumer_sync();
    return l;
}

template <typename WT>
__device__ void op_self_attention(const StepParams& p, const StepOp& op, int position, unsigned char* smem) {
    float* q = reinterpret_cast<float*>(smem);
    float* scratch = q + 64;
    float* fold = scratch + 8;
    float* result = fold + kFold;
    float* scores = result + 64;
    const int D = p.head_width;
    // A fused out-projection with CTAs to spare: `shares` CTAs a (row, head),
    // each attending in full (the same sums in the same order) and projecting
    // its share of the output tiles, so no CTA reads all of the head's
    // columns of the out-projection.
    const int pairs = p.rows * p.heads;
    const int shares = op.out_weight && pairs < (int)gridDim.x ? min((int)gridDim.x / pairs, (p.width + 15) / 16) : 1;
    for (int item = blockIdx.x; item < pairs * shares; item += gridDim.x) {
        const int share = item / pairs, r = (item % pairs) / p.heads, head = item % p.heads;
        const int b = r / p.tokens, t = r % p.tokens;
        const int keys = position + t + 1;
        Trace trs = trace_of(p.profile);
        trs.begin();
        consumer_sync();
        const WT* K = static_cast<const WT*>(op.keys) + (size_t)b * op.window_stride + (size_t)head * D;
        const WT* V = static_cast<const WT*>(op.values) + (size_t)b * op.window_stride + (size_t)head * D;
        float l;
        if (D == 64 && keys <= kThreads) {
            // Up to one key a thread: every key row and value piece of the item
            // is loaded with q, one round trip in all.
            l = self_item_in_registers<WT>(p, r, head, keys, K, V, op.key_stride, q, scratch, fold, result, scores);
        } else {
            for (int c = threadIdx.x; c < D; c += kThreads)
                q[c] = ld_cg(p.q + (size_t)r * p.width + head * D + c) * p.scale;
            consumer_sync();
            const float m = consumer_max(attention_scores<WT, false>(q, K, op.key_stride, D, 0, keys, scores), scratch);
            float local = 0.f;
            for (int j = threadIdx.x; j < keys; j += kThreads) {
                const float e = __expf(scores[j] - m);
                scores[j] = e;
                local += e;
            }
            l = consumer_sum(local, scratch);
            attention_values<WT, false>(scores, V, op.key_stride, D, 0, keys, fold, result);
        }
        trs.end(kTrSelf);
        if (op.out_weight) {
            // The head's out-projection share, from its 16-bit values (hi, lo).
            __shared__ __align__(16) WT attended[128];
            for (int c = threadIdx.x; c < 64; c += kThreads) store_split(attended + c, 64, result[c] / l);
            consumer_sync();
            head_out_projection<WT>(p, op, r, head, attended, share, shares);
            continue;
        }
        WT* out = static_cast<WT*>(p.attn16);
        for (int c = threadIdx.x; c < D; c += kThreads)
            store_split(out + act_index(p, r, head * D + c, p.kpd), lo_plane(p, p.kpd), result[c] / l);
    }
}

// Self attention with many rows: a warp per (row, head) item, so a CTA has
// kWarps items' loads in flight instead of one.  64-wide heads.  Scores:
// eight keys a pass, four lanes a key (32 bytes each, two shuffles to
// join), four passes' loads issued together; the weights in the warp's
// score row; values: four keys a pass, a 16-byte piece a lane, eight passes'
// loads together, the four key slots joined at the end.  Keys and values
// come through L2 (this launch's q/k/v op wrote the newest ones).


template <typename WT>
__device__ void self_attention_warps(const StepParams& p, const StepOp& op, int position, unsigned char* work) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = p.heads;
    float* sc = reinterpret_cast<float*>(work) + warp * kSelfWarpKeys;
    const int items = p.rows * H;
    for (int item = blockIdx.x * kWarps + warp; item < items; item += gridDim.x * kWarps) {
        const int r = item / H, head = item % H;
        const int b = r / p.tokens, t = r % p.tokens;
        const int keys = position + t + 1;
        const WT* K = static_cast<const WT*>(op.keys) + (size_t)b * op.window_stride + head * 64;
        const WT* V = static_cast<const WT*>(op.values) + (size_t)b * op.window_stride + head * 64;
        // This lane's quarter of q: dims 16*qd .. 16*qd + 15.
        const int slot = lane >> 2, qd = lane & 3;
        float q[16];
        const float* qrow = p.q + (size_t)r * p.width + head * 64 + 16 * qd;
        if (op.qkv_partial) {
            // The q/k/v product's join for this (row, head): its 192 rows'
            // partials (q, k, v: rows 192 head ..), three pairs a lane, every
            // split's loads in flight before the sums, which run in split
            // order and add the bias last, as the product's join would.  k and
            // v go to the caches at the row's position; q to this warp's
            // score row, which the scores overwrite later.
            const int S = op.qkv_splits;
            float2 sum[3] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
            for (int k0 = 0; k0 < S; k0 += kDeferLoads) {
                float2 v[kDeferLoads][3];
#pragma unroll
                for (int k = 0; k < kDeferLoads; ++k)
#pragma unroll
                    for (int j = 0; j < 3; ++j) {
                        const int n = head * 192 + 2 * (lane + 32 * j);
                        const float* at = op.qkv_partial + (size_t)(k0 + k) * op.qkv_split_stride +
                                          ((size_t)(n >> 7) * op.qkv_row_stride + r) * 128 + (n & 127);
                        v[k][j] = k0 + k < S ? __ldcg(reinterpret_cast<const float2*>(at)) : make_float2(0.f, 0.f);
                    }
#pragma unroll
                for (int k = 0; k < kDeferLoads; ++k)
                    if (k0 + k < S)
#pragma unroll
                        for (int j = 0; j < 3; ++j) {
                            sum[j].x += v[k][j].x;
                            sum[j].y += v[k][j].y;
                        }
            }
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                const int i = 2 * (lane + 32 * j), n = head * 192 + i;  // i: 0..191 within the head
                const float2 bias = __ldg(reinterpret_cast<const float2*>(op.qkv_bias + n));
                const float x = sum[j].x + bias.x, y = sum[j].y + bias.y;
                if (i < 64) {
                    sc[i] = x;
                    sc[i + 1] = y;
                } else {
                    WT* cache = const_cast<WT*>(i < 128 ? K : V) + (size_t)(position + t) * op.key_stride + (i & 63);
                    cache[0] = Half16<WT>::from_float(x);
                    cache[1] = Half16<WT>::from_float(y);
                }
            }
            __syncwarp();
            qrow = sc + 16 * qd;
        }
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
            const float4 v = op.qkv_partial ? *reinterpret_cast<const float4*>(qrow + i)
                                            : __ldcg(reinterpret_cast<const float4*>(qrow + i));
            q[i] = v.x * p.scale;
            q[i + 1] = v.y * p.scale;
            q[i + 2] = v.z * p.scale;
            q[i + 3] = v.w * p.scale;
        }
        // (The scores below overwrite the score row only after every lane
        // has its q.)
        __syncwarp();
        float mx = -INFINITY;
        for (int j0 = 0; j0 < keys; j0 += 32) {
            uint4 ka[4], kb[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int j = min(j0 + 8 * u + slot, keys - 1);
                const WT* row = K + (size_t)j * op.key_stride + 16 * qd;
                ka[u] = ld_cg4(row);
                kb[u] = ld_cg4(row + 8);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int j = j0 + 8 * u + slot;
                const float2 a0 = Half16<WT>::pair_to_float2(ka[u].x), a1 = Half16<WT>::pair_to_float2(ka[u].y);
                const float2 a2 = Half16<WT>::pair_to_float2(ka[u].z), a3 = Half16<WT>::pair_to_float2(ka[u].w);
                const float2 b0 = Half16<WT>::pair_to_float2(kb[u].x), b1 = Half16<WT>::pair_to_float2(kb[u].y);
                const float2 b2 = Half16<WT>::pair_to_float2(kb[u].z), b3 = Half16<WT>::pair_to_float2(kb[u].w);
                float part = q[0] * a0.x + q[1] * a0.y + q[2] * a1.x + q[3] * a1.y + q[4] * a2.x + q[5] * a2.y +
                             q[6] * a3.x + q[7] * a3.y;
                part += q[8] * b0.x + q[9] * b0.y + q[10] * b1.x + q[11] * b1.y + q[12] * b2.x + q[13] * b2.y +
                        q[14] * b3.x + q[15] * b3.y;
                part += __shfl_xor_sync(0xffffffffu, part, 1);
                part += __shfl_xor_sync(0xffffffffu, part, 2);
                if (j < keys) {
                    if (qd == 0) sc[j] = part;
                    mx = fmaxf(mx, part);
                }
            }
        }
        mx = warp_max(mx);
        __syncwarp();
        float l = 0.f;
        for (int j = lane; j < keys; j += 32) {
            const float e = __expf(sc[j] - mx);
            sc[j] = e;
            l += e;
        }
        l = warp_sum(l);
        __syncwarp();
        const int vslot = lane >> 3, piece = lane & 7;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int j0 = 0; j0 < keys; j0 += 32) {
            uint4 v[8];
            float w[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int j = j0 + 4 * u + vslot;
                const int jj = min(j, keys - 1);
                v[u] = ld_cg4(V + (size_t)jj * op.key_stride + 8 * piece);
                w[u] = j < keys ? sc[jj] : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float2 f0 = Half16<WT>::pair_to_float2(v[u].x), f1 = Half16<WT>::pair_to_float2(v[u].y);
                const float2 f2 = Half16<WT>::pair_to_float2(v[u].z), f3 = Half16<WT>::pair_to_float2(v[u].w);
                acc[0] += w[u] * f0.x;
                acc[1] += w[u] * f0.y;
                acc[2] += w[u] * f1.x;
                acc[3] += w[u] * f1.y;
                acc[4] += w[u] * f2.x;
                acc[5] += w[u] * f2.y;
                acc[6] += w[u] * f3.x;
                acc[7] += w[u] * f3.y;
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 8);
            acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 16);
        }
        if (vslot == 0) {
            WT* out = static_cast<WT*>(p.attn16);
            const float inv = 1.f / l;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                store_split(out + act_index(p, r, head * 64 + 8 * piece + i, p.kpd), lo_plane(p, p.kpd), acc[i] * inv);
        }
        __syncwarp();
    }
}

// ------------------------------------------------------- cross attention

// The keys and values of one (window, layer, head) are one contiguous block
// of encoder rows [K | V], 2D 16-bit values each, so `chunk` consecutive
// keys are one bulk copy: they stream through the ring like weights, and the
// producer fetches them while the ops before this one run.  An item (row,
// head, split) covers `span` chunks; CTA c takes items c, c + grid, ... and
// all its warps work on every chunk, each on its own keys: key j belongs to
// warp (j / 4) % kWarps.  Per chunk, a warp scores its keys, the CTA agrees
// on the running maximum (one barrier), each warp weights its keys' values,
// and the CTA folds the warps' sums (a second barrier) into an online
// softmax held by threads < D (SingleQueryAttention.h:11-37 joins splits the
// same way).  With several splits per (row, head) the last to finish joins
// the partials.

__device__ __forceinline__ int cross_units(const StepOp& op) { return (op.key_count + op.chunk - 1) / op.chunk; }
__device__ __forceinline__ int cross_item_units(const StepOp& op, int item, int units) {
    return max(0, min(op.span, units - (item % op.splits) * op.span));
}
// Key of this warp's i-th owned key slot (keys 4g..4g+3 for g = warp, warp + kWarps, ...).
__device__ __forceinline__ int owned_key(int warp, int i) { return 4 * (warp + kWarps * (i >> 2)) + (i & 3); }

// Scores of this warp's keys of the chunk into sc[] (lane per key); returns
// their maximum.  Heads other than 64 wide.
template <typename WT>
__device__ __forceinline__ float cross_scores(const WT* rows, int n, int D, const float* q, float* sc) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float mx = -INFINITY;
    for (int i = lane;; i += 32) {
        const int j = owned_key(warp, i);
        if (j >= n) break;
        const WT* k = rows + (size_t)j * 2 * D;
        float sum = 0.f;
        for (int c = 0; c < D; c += 2) {
            const float2 f = Half16<WT>::pair_to_float2(*reinterpret_cast<const uint32_t*>(k + c));
            sum += q[c] * f.x + q[c + 1] * f.y;
        }
        sc[j] = sum;
        mx = fmaxf(mx, sum);
    }
    return warp_max(mx);
}

// exp(sc[j] - m) for this warp's keys, written back; returns their sum.
__device__ __forceinline__ float cross_weights(int n, float m, float* sc) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float sum = 0.f;
    for (int i = lane;; i += 32) {
        const int j = owned_key(warp, i);
        if (j >= n) break;
        const float e = __expf(sc[j] - m);
        sc[j] = e;
        sum += e;
    }
    __syncwarp();
    return warp_sum(sum);
}

// sum over this warp's keys of sc[j] V[j] into a[2]: lane l holds channels
// l and l + 32.  Heads other than 64 wide.
template <typename WT>
__device__ __forceinline__ void cross_values(const WT* rows, int n, int D, const float* sc, float (&a)[2]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    a[0] = a[1] = 0.f;
    for (int i = 0;; ++i) {
        const int j = owned_key(warp, i);
        if (j >= n) break;
        const WT* v = rows + (size_t)j * 2 * D + D;
        const float w = sc[j];
        if (lane < D) a[0] += w * Half16<WT>::to_float(v[lane]);
        if (lane + 32 < D) a[1] += w * Half16<WT>::to_float(v[lane + 32]);
    }
}

// The last split of a (row, head), one warp: joins the splits' partials
// [max, sum, D values] with every load of a lane in flight at once.
// `staged`: the partials already in shared memory (a cooperative join).
__device__ __forceinline__ float join_load(const float* at, bool staged) {
    return staged ? *at : ld_cg(at);
}
template <typename WT>
__device__ void cross_join(const StepParams& p, const StepOp& op, int r, int head, WT* to_shared = nullptr,
                           const float* staged = nullptr) {
    const int lane = threadIdx.x & 31;
    const int D = p.head_width, S = op.splits;
    const bool sh = staged != nullptr;
    const float* part = sh ? staged : p.partial + ((size_t)r * p.heads + head) * S * (D + 2);
    const float m_own = lane < S ? join_load(part + (size_t)lane * (D + 2), sh) : -INFINITY;
    const float l_own = lane < S ? join_load(part + (size_t)lane * (D + 2) + 1, sh) : 0.f;
    const float mx = warp_max(m_own);
    const float f_own = m_own == -INFINITY ? 0.f : __expf(m_own - mx);
    const float l = warp_sum(l_own * f_own);
    float o[2] = {0.f, 0.f};
    const int c0 = lane, c1 = lane + 32;
#pragma unroll 8
    for (int sp = 0; sp < S; ++sp) {
        const float f = __shfl_sync(0xffffffffu, f_own, sp);
        const float* ps = part + (size_t)sp * (D + 2) + 2;
        if (c0 < D) o[0] += join_load(ps + c0, sh) * f;
        if (c1 < D) o[1] += join_load(ps + c1, sh) * f;
    }
    const float a0 = o[0] / l + (op.value_bias && c0 < D ? __ldg(op.value_bias + head * D + c0) : 0.f);
    const float a1 = o[1] / l + (op.value_bias && c1 < D ? __ldg(op.value_bias + head * D + c1) : 0.f);
    if (to_shared) {
        // A fused out-projection reads the 16-bit values (hi, then lo 64 on)
        // from shared memory.
        if (c0 < D) store_split(to_shared + c0, 64, a0);
        if (c1 < D) store_split(to_shared + c1, 64, a1);
        return;
    }
    WT* out = static_cast<WT*>(p.attn16);
    if (c0 < D) store_split(out + act_index(p, r, head * D + c0, p.kpd), lo_plane(p, p.kpd), a0);
    if (c1 < D) store_split(out + act_index(p, r, head * D + c1, p.kpd), lo_plane(p, p.kpd), a1);
}

// Shared memory: [q: 64][max: 2 x 8][sum: 2 x 8][fold: 2 x kWarps x 64][scores: kMaxCrossUnitKeys]
template <typename WT>
__device__ void cross_attention_cores(const StepParams& p, const StepOp& op, Stream& s, unsigned char* work) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int D = p.head_width, H = p.heads, S = op.splits;
    const int units = cross_units(op);
    const int items = p.rows * H * S;
    float* q = reinterpret_cast<float*>(work);
    float* wmax = q + 64;
    float* wsum = wmax + 16;
    float* fold = wsum + 16;
    float* sc = fold + 2 * kWarps * 64;
    __shared__ int is_last;
    int par = 0;
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int split = item % S, head = (item / S) % H, r = item / (S * H);
        const int count = cross_item_units(op, item, units);
        consumer_sync();
        for (int c = threadIdx.x; c < D; c += kThreads) q[c] = ld_cg(p.q + (size_t)r * p.width + head * D + c) * p.scale;
        consumer_sync();
        float m_run = -INFINITY, l_run = 0.f, o_run = 0.f;  // o_run: channel threadIdx.x < D
        for (int t = 0; t < count; ++t) {
            const WT* rows = reinterpret_cast<const WT*>(acquire_unit(p, s));
            const int k0 = (split * op.span + t) * op.chunk;
            const int n = min(op.chunk, op.key_count - k0);
            Trace tr = trace_of(p.profile);
            tr.begin();
            const float wm = cross_scores<WT>(rows, n, D, q, sc);
            if (lane == 0) wmax[par * 8 + warp] = wm;
            consumer_sync();
            float cm = -INFINITY;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) cm = fmaxf(cm, wmax[par * 8 + w]);
            const float m_new = fmaxf(m_run, cm);
            const float keep = m_run == -INFINITY ? 0.f : __expf(m_run - m_new);
            const float ws = cross_weights(n, m_new, sc);
            float a[2];
            cross_values<WT>(rows, n, D, sc, a);
            release_unit(s);
            if (lane < D) fold[(par * kWarps + warp) * 64 + lane] = a[0];
            if (lane + 32 < D) fold[(par * kWarps + warp) * 64 + lane + 32] = a[1];
            if (lane == 0) wsum[par * 8 + warp] = ws;
            consumer_sync();
            float l_chunk = 0.f, o_chunk = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) l_chunk += wsum[par * 8 + w];
            if (threadIdx.x < D) {
#pragma unroll
                for (int w = 0; w < kWarps; ++w) o_chunk += fold[(par * kWarps + w) * 64 + threadIdx.x];
            }
            o_run = o_run * keep + o_chunk;
            l_run = l_run * keep + l_chunk;
            m_run = m_new;
            par ^= 1;
            tr.end(kTrAttention);
        }
        if (S == 1) {
            if (threadIdx.x < D)
                store_split(static_cast<WT*>(p.attn16) + act_index(p, r, head * D + threadIdx.x, p.kpd),
                            lo_plane(p, p.kpd),
                            o_run / l_run + (op.value_bias ? __ldg(op.value_bias + head * D + threadIdx.x) : 0.f));
            continue;
        }
        float* part = p.partial + (((size_t)r * H + head) * S + split) * (D + 2);
        if (threadIdx.x < D) part[2 + threadIdx.x] = o_run;
        if (threadIdx.x == 0) {
            part[0] = m_run;
            part[1] = l_run;
        }
        consumer_sync();
        if (threadIdx.x == 0) {
            unsigned* counter = p.combine_counters + (size_t)r * H + head;
            is_last = arrive_acq_rel(counter) == (unsigned)(S - 1);
            if (is_last) atomicExch(counter, 0u);
        }
        consumer_sync();
        if (is_last && warp == 0) cross_join<WT>(p, op, r, head);
    }
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&d)[4], const void* row) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(smem_address(row))
                 : "memory");
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&d)[4], const void* row) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(smem_address(row))
                 : "memory");
}

// Shared memory of cross_attention_mma before a fused query's tile:
// [q: 64][warp max: 8][warp sum: 8][warp rows: kWarps x 64] floats.
constexpr int kCrossQueryOffset = 2304;

// A fused cross query (op.gamma set: a few rows): q of (row r, head) is
// LN2(h_r) . Wq[64 head .. 64 head + 63]^T + bq, scaled by 1/sqrt(D)
// (Decoder.cpp:93-100, DecoderShape.cpp:19-26), computed by the item itself
// instead of by a product op of its own.  The LayerNorm prologue adds the
// self attention's out-projection partials (its residual, Decoder.cpp:80-91);
// keep_sum: this CTA stores the sums as the new residual rows.  The head's
// four 16-row weight tiles come off the weight stream ahead of the item's
// keys.  Work area at `area`: [xs: 2 planes x 8 x pitch 16-bit]; after the
// query, the same area holds a cooperative join's partials (kMaxCrossSplits
// x 66 floats).
template <typename WT>
__device__ bool cross_query(const StepParams& p, const StepOp& op, int r, int head, bool keep_sum, Stream& s,
                            unsigned char* area, float* q) {
    const int pitch = tile_pitch(p.kpd), D = p.head_width;
    WT* xs = reinterpret_cast<WT*>(area);
    // The q biases of this lane's two rows, loaded with the LayerNorm's rows.
    const int tiles = round16(D) / 16, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qn = 16 * warp + (lane >> 2);
    const float* qbias = op.bias + head * round16(D);
    const float bias_a = warp < tiles && qn < D ? __ldg(qbias + qn) : 0.f;
    const float bias_b = warp < tiles && qn + 8 < D ? __ldg(qbias + qn + 8) : 0.f;
    Addends add;
    if (op.addend_count > 0)
        add = Addends{op.addends, op.addend_count, op.addend_stride, op.addend_bias, keep_sum ? op.sum_out : nullptr};
    layer_norm_tile<WT>(p, op.norm_input ? op.norm_input : p.h, op.gamma, op.beta, r, 1, 1, 0, xs, pitch,
                        (size_t)8 * pitch, nullptr, add);
    consumer_sync();
    // Warp j < tiles owns q tile j (one unit: a stage holds a whole tile)
    // over all of K, so no partial sums cross warps.  (Spreading the tiles'
    // chunks over all seven warps, with a reduction after, measured slower:
    // each warp then waits for every tile.)
    if (warp < tiles) {
        const unsigned long long index = s.next + warp;
        const unsigned char* unit = owned_unit_at(p, s, index);
        float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
        const bool x_ok[1] = {(lane >> 2) == 0};
        chunks_product<WT, 1, true>(unit, 0, 1, op.kp / 32, xs, pitch, (size_t)8 * pitch, 0, x_ok, acc);
        release_at(s, index, kWarps);
        // Column 0 (the one row) sits in lanes t == 0: q rows g and g + 8 of the tile.
        if ((lane & 3) == 0) {
            if (qn < D) q[qn] = (acc[0][0] + bias_a) * p.scale;
            if (qn + 8 < D) q[qn + 8] = (acc[0][2] + bias_b) * p.scale;
        }
    }
    s.next += tiles;
    // (A wait that gave up hands back its stage all the same; the kernel
    // leaves at the next grid barrier.)
    return true;
}

// One warp's 16-key group n0 of a cross unit (rows: the unit's keys in
// the rotated layout, n of them) against q (qa: q's hi + lo halves as rows 0
// and 1 of A): scores as m16n8k16 products with the keys as B, loaded by
// ldmatrix.  Lanes 0..7 end with the scores of keys n0 + 2t, n0 + 2t + 1,
// n0 + 8 + 2t, n0 + 9 + 2t (t = lane % 4) in v[0..3]; -inf past n, off
// those lanes, or for a group at or past n.
template <typename WT>
__device__ __forceinline__ void cross_group_scores(const WT* rows, int n, int n0, const uint32_t (&qa)[4][2],
                                                   float (&v)[4]) {
    const int lane = threadIdx.x & 31, t4 = lane & 3, mi = lane >> 3, rr = lane & 7;
    const bool row0 = lane < 4, pair = lane < 8;
    if (n0 >= n) {
        v[0] = v[1] = v[2] = v[3] = -INFINITY;
        return;
    }
    // Even and odd key pieces accumulate apart: four chains of two products.
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
    float t0[4] = {0.f, 0.f, 0.f, 0.f}, t1[4] = {0.f, 0.f, 0.f, 0.f};
    {
        // Keys n0 + 8*(mi/2) + rr, key pieces 2kk + mi%2 (rows past the
        // unit's keys read its last key; their scores are dropped).
        const int key = min(n0 + 8 * (mi >> 1) + rr, n - 1);
        uint32_t b[4][4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
            ldmatrix_x4(b[kk], rows + (size_t)key * 128 + cross_piece(2 * kk + (mi & 1), key) * 8);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const uint32_t a[4] = {qa[kk][0], 0u, qa[kk][1], 0u};
            const uint32_t b0[2] = {b[kk][0], b[kk][1]}, b1[2] = {b[kk][2], b[kk][3]};
            mma_16816<WT>(kk & 1 ? t0 : s0, a, b0);
            mma_16816<WT>(kk & 1 ? t1 : s1, a, b1);
        }
    }
    // Rows 0 (hi, lanes 0..3) and 1 (lo, lanes 4..7): keys n0+2t, n0+2t+1
    // (s0) and n0+8+2t, n0+9+2t (s1).  Their sum reaches lanes 0..7 alike.
    float sc[4] = {s0[0] + t0[0], s0[1] + t0[1], s1[0] + t1[0], s1[1] + t1[1]};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float other = __shfl_xor_sync(0xffffffffu, sc[i], 4);
        sc[i] = row0 ? sc[i] + other : other + sc[i];
    }
    const int ka = n0 + 2 * t4;
    v[0] = pair && ka < n ? sc[0] : -INFINITY;
    v[1] = pair && ka + 1 < n ? sc[1] : -INFINITY;
    v[2] = pair && ka + 8 < n ? sc[2] : -INFINITY;
    v[3] = pair && ka + 9 < n ? sc[3] : -INFINITY;
}

// o += P . V for the group's weights e (as cross_group_scores lays them
// out): P's hi half as row 0 of A, its lo half as row 1, the values as B by
// ldmatrix.trans.  Lanes 0..3 (row 0) and 4..7 (row 1) hold channels
// 8i + 2t, 8i + 2t + 1 in o[i]; the two rows add once per item.
template <typename WT>
__device__ __forceinline__ void cross_group_values(const WT* rows, int n, int n0, const float (&e)[4],
                                                   float (&o)[8][4]) {
    const int lane = threadIdx.x & 31, mi = lane >> 3, rr = lane & 7;
    const bool row0 = lane < 4, pair = lane < 8;
    uint32_t ph0, pl0, ph2, pl2;
    split_pair<WT>(e[0], e[1], ph0, pl0);
    split_pair<WT>(e[2], e[3], ph2, pl2);
    const uint32_t a[4] = {pair ? (row0 ? ph0 : pl0) : 0u, 0u, pair ? (row0 ? ph2 : pl2) : 0u, 0u};
    // Keys n0 + 8*(mi%2) + rr, value pieces 8 + 2cc + mi/2.
    const int key = min(n0 + 8 * (mi & 1) + rr, n - 1);
    uint32_t b[4][4];
#pragma unroll
    for (int cc = 0; cc < 4; ++cc)
        ldmatrix_x4_trans(b[cc], rows + (size_t)key * 128 + cross_piece(8 + 2 * cc + (mi >> 1), key) * 8);
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
        const uint32_t b0[2] = {b[cc][0], b[cc][1]}, b1[2] = {b[cc][2], b[cc][3]};
        mma_16816<WT>(o[2 * cc], a, b0);
        mma_16816<WT>(o[2 * cc + 1], a, b1);
    }
}

// 64-wide heads on the tensor cores.  A warp takes the unit's 16-key groups
// 16*warp, 16*(warp + kWarps), ...:
//   scores  m16n8k16 with q as row 0 of A (split hi + lo, so the product
//           carries nearly fp32 q) and B = the keys, loaded by ldmatrix from
//           rows whose pieces cross_piece rotates -- conflict-free;
//   values  row 0 of A = the weights p (hi + lo), which the score fragments
//           already hold in A's order, and B = the values by ldmatrix.trans.
// Lanes 0..3 carry row 0: the scores of keys 2t, 2t+1 (and + 8), and
// channels 8i+2t, 8i+2t+1 of the output.  Each warp keeps its own online
// softmax over the item; the warps join once per item.
// Shared memory: [q: 64][warp max: 8][warp sum: 8][warp rows: kWarps x 64]
// [the queries of the CTA's first kCrossQueryBatch items: 64 each]
constexpr int kCrossQueryBatch = 32;
// Stages of the weight-stream ring from which the cross attention takes its
// units two at a time (it holds two while the rest land).
constexpr int kCrossPairStages = 3;

template <typename WT>
__device__ void cross_attention_mma(const StepParams& p, const StepOp& op, Stream& s, unsigned char* work,
                                    unsigned use) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t4 = lane & 3;
    const bool row0 = lane < 4, pair = lane < 8;
    const int H = p.heads, S = op.splits;
    const int units = cross_units(op);
    const int items = p.rows * H * S;
    // A fused out-projection with every item on a CTA of its own: the
    // splits join together (below) instead of the last to finish alone.
    const bool cooperative = op.out_weight != nullptr && S > 1 && items <= (int)gridDim.x;
    // The op's fields in registers: the op list is in global memory, and the
    // ring's waits (asm with memory clobbers) would have them re-read.
    const int span = op.span, chunk = op.chunk, key_count = op.key_count;
    float* const q_home = reinterpret_cast<float*>(work);
    float* q = q_home;
    float* wmax = q_home + 64;
    float* wsum = wmax + 8;
    float* wrows = wsum + 8;
    float* qbatch = wrows + kWarps * 64;
    __shared__ int is_last;
    __shared__ __align__(16) WT attended[128];  // a fused out-projection's input (hi, lo)
    // The queries the previous op wrote, for the CTA's first items at once:
    // one round trip for the op rather than one an item.
    if (!op.gamma) {
        const int mine = min(kCrossQueryBatch, (items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x);
        for (int i = threadIdx.x; i < mine * 64; i += kThreads) {
            const int item = blockIdx.x + (i >> 6) * gridDim.x;
            const int head = (item / S) % H, r = item / (S * H);
            qbatch[i] = ld_cg(p.q + (size_t)r * p.width + head * 64 + (i & 63)) * p.scale;
        }
    }
    int nth = 0;  // this item's place among the CTA's items
    for (int item = blockIdx.x; item < items; item += gridDim.x, ++nth) {
        const int split = item % S, head = (item / S) % H, r = item / (S * H);
        const int count = cross_item_units(op, item, units);
        consumer_sync();
        q = q_home;
        if (op.gamma) {
            // The item's own query; item (r, head 0, split 0) keeps row r's residual sums.
            Trace trq = trace_of(p.profile);
            trq.begin();
            if (!cross_query<WT>(p, op, r, head, head == 0 && split == 0, s, work + kCrossQueryOffset, q)) return;
            trq.end(kTrQuery);
        } else if (nth < kCrossQueryBatch) {
            q = qbatch + 64 * nth;
        } else if (threadIdx.x < 64) {
            q[threadIdx.x] = ld_cg(p.q + (size_t)r * p.width + head * 64 + threadIdx.x) * p.scale;
        }
        consumer_sync();
        // Row 0 of A is q's hi half, row 1 its lo half (lanes 4..7), so one
        // product gives both, and the two rows add after the chain.
        uint32_t qa[4][2];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            if (pair) {
                uint32_t h0, l0, h1, l1;
                split_pair<WT>(q[16 * kk + 2 * t4], q[16 * kk + 2 * t4 + 1], h0, l0);
                split_pair<WT>(q[16 * kk + 2 * t4 + 8], q[16 * kk + 2 * t4 + 9], h1, l1);
                qa[kk][0] = row0 ? h0 : l0;
                qa[kk][1] = row0 ? h1 : l1;
            } else {
                qa[kk][0] = qa[kk][1] = 0u;
            }
        }
        float m_w = -INFINITY, l_w = 0.f;
        float o[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
        // Two units at a time (with three stages or more, so one more lands
        // meanwhile): each warp takes its 16-key group(s) in both, the scores
        // of both before one softmax update, then both groups' values --
        // twice the independent work between the dependent steps of one
        // group (its shuffles, its exponentials).  Measured a layer, one
        // unit at a time against two: medium.en at 64 windows 118 against 96
        // us, large-v3 at 128 windows 295 against 259.
        const int per = s.stages >= kCrossPairStages ? 2 : 1;
        for (int t = 0; t < count; t += per) {
            const bool two = per == 2 && t + 1 < count;
            const WT* ra = reinterpret_cast<const WT*>(unit_at(p, s, s.next));
            const WT* rb = two ? reinterpret_cast<const WT*>(unit_at(p, s, s.next + 1)) : ra;
            const int k0 = (split * span + t) * chunk;
            const int na = min(chunk, key_count - k0);
            const int nb = two ? min(chunk, key_count - k0 - chunk) : 0;
            Trace tr = trace_of(p.profile);
            tr.begin();
            for (int n0 = 16 * warp; n0 < max(na, nb); n0 += 16 * kWarps) {
                float va[4], vb[4];
                cross_group_scores<WT>(ra, na, n0, qa, va);
                cross_group_scores<WT>(rb, nb, n0, qa, vb);
                float gm = fmaxf(fmaxf(fmaxf(va[0], va[1]), fmaxf(va[2], va[3])),
                                 fmaxf(fmaxf(vb[0], vb[1]), fmaxf(vb[2], vb[3])));
                gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, 1));
                gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, 2));
                gm = __shfl_sync(0xffffffffu, gm, 0);
                const float m_new = fmaxf(m_w, gm);
                const float keep = m_w == -INFINITY ? 0.f : __expf(m_w - m_new);
                float ea[4], eb[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    ea[i] = va[i] == -INFINITY ? 0.f : __expf(va[i] - m_new);
                    eb[i] = vb[i] == -INFINITY ? 0.f : __expf(vb[i] - m_new);
                }
                float ls = ((ea[0] + ea[1]) + (ea[2] + ea[3])) + ((eb[0] + eb[1]) + (eb[2] + eb[3]));
                ls += __shfl_xor_sync(0xffffffffu, ls, 1);
                ls += __shfl_xor_sync(0xffffffffu, ls, 2);
                ls = __shfl_sync(0xffffffffu, ls, 0);
                l_w = l_w * keep + ls;
                m_w = m_new;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    o[i][0] *= keep;
                    o[i][1] *= keep;
                }
                if (n0 < na) cross_group_values<WT>(ra, na, n0, ea, o);
                if (n0 < nb) cross_group_values<WT>(rb, nb, n0, eb, o);
            }
            tr.end(kTrAttention);
            release_at(s, s.next);
            if (two) release_at(s, s.next + 1);
            s.next += two ? 2 : 1;
        }
        // Rows 0 and 1 of the output (P's hi and lo halves) add; then the
        // warps' softmaxes join.
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            o[i][0] += __shfl_xor_sync(0xffffffffu, o[i][0], 4);
            o[i][1] += __shfl_xor_sync(0xffffffffu, o[i][1], 4);
        }
        if (lane == 0) {
            wmax[warp] = m_w;
            wsum[warp] = l_w;
        }
        if (row0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                wrows[warp * 64 + 8 * i + 2 * t4] = o[i][0];
                wrows[warp * 64 + 8 * i + 2 * t4 + 1] = o[i][1];
            }
        }
        consumer_sync();
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wmax[w]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float f = wmax[w] == -INFINITY ? 0.f : __expf(wmax[w] - M);
            L += wsum[w] * f;
            if (threadIdx.x < 64) O += wrows[w * 64 + threadIdx.x] * f;
        }
        if (S == 1) {
            const float a = O / L + (op.value_bias ? __ldg(op.value_bias + head * 64 + (threadIdx.x & 63)) : 0.f);
            if (op.out_weight) {
                if (threadIdx.x < 64) store_split(attended + threadIdx.x, 64, a);
                consumer_sync();
                head_out_projection<WT>(p, op, r, head, attended);
                continue;
            }
            if (threadIdx.x < 64)
                store_split(static_cast<WT*>(p.attn16) + act_index(p, r, head * 64 + threadIdx.x, p.kpd),
                            lo_plane(p, p.kpd), a);
            continue;
        }
        Trace trj = trace_of(p.profile);
        trj.begin();
        float* part = p.partial + (((size_t)r * H + head) * S + split) * 66;
        if (threadIdx.x < 64) part[2 + threadIdx.x] = O;
        if (threadIdx.x == 0) {
            part[0] = M;
            part[1] = L;
        }
        consumer_sync();
        if (cooperative) {
            // Every split of the (row, head) joins: the splits meet at the
            // pair's counter (monotonic over the launch: `use` cross ops have
            // passed it before this one), each joins the partials itself --
            // the same sums in the same order as a single joiner -- and
            // projects its share of the output tiles.  Each split is the one
            // item of its CTA and every CTA is resident, so all of them
            // arrive; the wait is bounded all the same.
            if (threadIdx.x == 0) {
                unsigned* counter = p.combine_counters + (size_t)r * H + head;
                asm volatile("red.release.gpu.global.add.u32 [%0], %1;\n" ::"l"(counter), "r"(1u) : "memory");
                const unsigned target = (unsigned)S * (use + 1u);
                const unsigned long long start = global_ns();
                int ok = 1;
                for (unsigned spin = 1; ld_acquire(counter) < target; ++spin) {
                    if ((spin & 15) != 0) continue;
                    if (ld_volatile(p.state + kAbort)) { ok = 0; break; }
                    if (global_ns() - start > kWaitTimeoutNs) {
                        record_timeout(p, kWaitJoin, (long long)item);
                        ok = 0;
                        break;
                    }
                }
                is_last = ok;
            }
            consumer_sync();
            if (!is_last) return;
            // Every split's partial into shared memory with all of them in
            // flight at once (the query's tile is free by now): one round
            // trip to L2, where a warp reading them in turn takes several.
            {
                constexpr int kPer = (kMaxCrossSplits * 66 + kThreads - 1) / kThreads;
                float* staged = reinterpret_cast<float*>(work + kCrossQueryOffset);
                const float* from = p.partial + ((size_t)r * H + head) * S * 66;
                float v[kPer];
#pragma unroll
                for (int k = 0; k < kPer; ++k) {
                    const int i = threadIdx.x + k * kThreads;
                    v[k] = i < S * 66 ? ld_cg(from + i) : 0.f;
                }
#pragma unroll
                for (int k = 0; k < kPer; ++k) {
                    const int i = threadIdx.x + k * kThreads;
                    if (i < S * 66) staged[i] = v[k];
                }
                consumer_sync();
                if (warp == 0) cross_join<WT>(p, op, r, head, attended, staged);
            }
            consumer_sync();
            trj.end(kTrJoin);
            head_out_projection<WT>(p, op, r, head, attended, split, S);
            continue;
        }
        if (threadIdx.x == 0) {
            unsigned* counter = p.combine_counters + (size_t)r * H + head;
            is_last = arrive_acq_rel(counter) == (unsigned)(S - 1);
            if (is_last) atomicExch(counter, 0u);
        }
        consumer_sync();
        if (is_last) {
            if (warp == 0) cross_join<WT>(p, op, r, head, op.out_weight ? attended : nullptr);
            if (op.out_weight) {
                consumer_sync();
                trj.end(kTrJoin);
                head_out_projection<WT>(p, op, r, head, attended);
            }
        } else {
            trj.end(kTrJoin);
        }
    }
}

template <typename WT>
__device__ void op_cross_attention(const StepParams& p, const StepOp& op, Stream& s, unsigned char* work,
                                   unsigned use) {
    if (p.head_width == 64) cross_attention_mma<WT>(p, op, s, work, use);
    else cross_attention_cores<WT>(p, op, s, work);
}

// ----------------------------------------------------------- L2 prefetch

// The weight stream moves ~100 MB or more a step through L2, so data read
// straight from memory a step after it was last touched has left L2 by
// then, and each such read would cost its op a DRAM round trip on the
// critical path.  Static data (parameters, a fused out-projection's columns,
// the mask) is prefetched by the producer warp from the schedule; what
// depends on the position is prefetched here by thread 0, from fields of the
// op it is already running: during the logits, the next step's position
// rows; during a q/k/v product that asks for it (a few rows), the self keys
// and values 0 .. position + T - 1 its self attention will read, 4 KB a CTA.
__device__ void prefetch_rows(const StepParams& p, const StepOp& op, int position) {
    const unsigned cta = blockIdx.x, grid = gridDim.x;
    if (op.kind == kOpLogits) {
        if (cta == 0 && position + 2 * p.tokens <= p.max_positions)
            prefetch_l2(p.position_table + (size_t)(position + p.tokens) * p.width,
                        (unsigned long long)p.tokens * p.width * 4);
        return;
    }
    if (op.kind != kOpProduct || !op.prefetch_keys) return;
    const unsigned long long bytes = (unsigned long long)(position + p.tokens) * p.width * 2;
    const unsigned long long per = (bytes + 4095) / 4096;
    const unsigned long long window = (unsigned long long)p.max_positions * p.width * 2;
    for (unsigned long long i = cta; i < 2ull * (unsigned long long)p.windows * per; i += grid) {
        const unsigned long long which = i / per, o = (i % per) * 4096;
        const unsigned char* base = static_cast<const unsigned char*>((which & 1) ? op.self_values : op.self_keys);
        prefetch_l2(base + (which >> 1) * window + o, bytes - o < 4096 ? bytes - o : 4096);
    }
}

// -------------------------------------------------------------- the kernel

constexpr int kMaxStages = kMaxStreamStages;

// Consumers leave together; warp 0 frees the tensor memory (every product
// that wrote it has completed: each item waited for its commit).
__device__ __forceinline__ void release_tensor_memory(const StepParams& p, const TensorMemory& tm) {
    if (!p.umma) return;
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    consumer_sync();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (threadIdx.x < 32)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm.base), "r"(kTmemColumns));
}

// UMMA: the tensor-core product path (p.umma); a separate instantiation, so
// the mma.sync kernel carries none of it.
template <typename WT, int NT, bool UMMA>
__global__ void __launch_bounds__(kBlockThreads, 1) decode_kernel(StepParams p) {
    extern __shared__ __align__(128) unsigned char dynamic_smem[];
    __shared__ int stop_flag;
    __shared__ unsigned long long armed_units;
    __shared__ uint32_t tmem_slot;
    __shared__ __align__(8) uint64_t tmem_done;
    __shared__ __align__(8) uint64_t x_full[kMaxXStages];
    __shared__ __align__(8) uint64_t x_empty[kMaxXStages];
    // The tensor-core kernel's ring starts on a 1024-byte boundary (the
    // 128-byte swizzle's period).  The mma.sync kernel keeps the 128-byte
    // start: aligning it too measured 6 % slower at 32 windows.
    unsigned char* smem = UMMA ? reinterpret_cast<unsigned char*>(
                                     (reinterpret_cast<uintptr_t>(dynamic_smem) + 1023) & ~static_cast<uintptr_t>(1023))
                               : dynamic_smem;
    Stream s;
    s.stages = p.stages;
    s.div.set(p.stages);
    s.stage_bytes = p.stage_bytes;
    s.ring = smem;
    s.full = reinterpret_cast<uint64_t*>(smem + (size_t)s.stages * s.stage_bytes);
    s.empty = s.full + kMaxStages;
    unsigned char* work = smem + (size_t)s.stages * s.stage_bytes + 16 * kMaxStages;
    s.next = 0;
    s.armed = &armed_units;
    if (threadIdx.x == 0) {
        stop_flag = 0;
        armed_units = 0;
        for (int i = 0; i < kTrSections; ++i) trace_cycles[i] = 0;
        for (int i = 0; i < s.stages; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_address(s.full + i)) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_address(s.empty + i)), "r"(kWarps)
                         : "memory");
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_address(&tmem_done)) : "memory");
        for (int i = 0; i < kMaxXStages; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_address(x_full + i)) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_address(x_empty + i)) : "memory");
        }
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (UMMA && threadIdx.x < 32) {
        __syncwarp();  // tcgen05.alloc is warp-collective; lane 0 has just set up the barriers
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_address(&tmem_slot)),
                     "r"(kTmemColumns));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (UMMA) asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (UMMA) asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    TensorMemory tm{UMMA ? tmem_slot : 0u, &tmem_done, 0u,
                    reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(work) + 1023) &
                                                     ~static_cast<uintptr_t>(1023)),
                    x_full, x_empty, p.umma_x_stages, p.umma_x_stage_bytes, 0ull, RingDivisor{}};
    tm.x_div.set(p.umma_x_stages >= 2 ? p.umma_x_stages : 2);  // (unused without the tcgen05 products)
    volatile int* stop = &stop_flag;
    if (threadIdx.x >= kConsumers) {
        if (threadIdx.x == kConsumers) produce(p, s, stop);
        return;
    }

    unsigned epoch = 0;
    __shared__ __align__(16) StepOp op_slot[2];
    copy_op(p.ops, op_slot, (int)threadIdx.x);
    consumer_sync();
    int slot = 0;
    unsigned cross_uses = 0;  // cross-attention ops run so far in this launch
    const bool stamp = p.profile != nullptr && blockIdx.x == 0 && threadIdx.x == 0;
    for (int step = 0; step < p.steps; ++step) {
        const int position = ld_volatile(p.state + kPosition);
        if (stamp && step == 0) p.profile[0] = global_ns();
        for (int i = 0; i < p.n_ops; ++i) {
            const StepOp& op = op_slot[slot];
            if (threadIdx.x == 0) prefetch_rows(p, op, position);
            Trace tro = trace_of(p.profile);
            tro.begin();
            switch (op.kind) {
            case kOpEmbed: op_embed<WT>(p, position); break;
            case kOpProduct:
                if constexpr (UMMA) product_umma<WT>(p, op, position, step, i, s, tm);
                else op_product<WT, NT>(p, op, position, s, work);
                break;
            case kOpSelfAttention:
                // As many items as CTAs or more: a warp per item; fewer: the
                // whole CTA on each.
                if (!op.out_weight && p.head_width == 64 && p.max_positions <= kSelfWarpKeys &&
                    p.rows * p.heads >= (int)gridDim.x)
                    self_attention_warps<WT>(p, op, position, work);
                else
                    op_self_attention<WT>(p, op, position, work);
                break;
            case kOpCrossAttention: op_cross_attention<WT>(p, op, s, work, cross_uses++); break;
            case kOpLogits: {
                Trace trl = trace_of(p.profile);
                trl.begin();
                if constexpr (UMMA)
                    logits_umma<WT>(p, op, position, s, tm);
                else
                    op_logits<WT, NT>(p, op, position, s, work);
                trl.end(kTrLogits);
                break;
            }
            case kOpNorm: op_norm<WT>(p, op, work); break;
            }
            tro.end(kTrOther);
            Trace trb = trace_of(p.profile);
            trb.begin();
            const bool passed = grid_barrier(p, epoch, p.ops + (i + 1 < p.n_ops ? i + 1 : 0), op_slot + (slot ^ 1));
            slot ^= 1;
            trb.end(kTrBarrier);
            if (!passed) {
                trace_flush(p);
                if (threadIdx.x == 0) *stop = 1;
                if (UMMA) release_tensor_memory(p, tm);
                return;
            }
            if (stamp && step == 0) p.profile[i + 1] = global_ns();
        }
        if (p.stop_enabled && ld_volatile(p.state + kAllEnded)) break;
    }
    trace_flush(p);
    if (threadIdx.x == 0) *stop = 1;
    if (UMMA) release_tensor_memory(p, tm);
}

// Shared memory past the ring: the largest work area any op of the launch uses.
template <typename WT, int NT>
size_t work_bytes(const StepParams& p, int max_chunk) {
    constexpr int RT = 8 * NT;
    const size_t product = (size_t)2 * RT * tile_pitch(p.kpd) * sizeof(WT) +
                           sizeof(float) * (kWarps * 16 * RT + 16 * RT) + (size_t)p.out_rows * 8 +
                           sizeof(float) * 2 * kWarps * RT;
    const size_t attention =
        sizeof(float) * std::max<size_t>({(size_t)kAttentionFixed + std::max(max_chunk, p.max_positions),
                                          (size_t)(64 + 32 + 2 * kWarps * 64 + kMaxCrossUnitKeys),
                                          (size_t)(64 + 16 + kWarps * 64 + kCrossQueryBatch * 64),
                                          (size_t)kWarps * kSelfWarpKeys});
    size_t work;
    if (p.umma) {
        // Tensor-core products and logits: the activation ring (1024-byte
        // aligned), the logits' per-row best and tile scratch past it; a
        // norm op's row (both planes).
        const size_t ring = (size_t)1024 + std::max((size_t)p.umma_x_stages * p.umma_x_stage_bytes,
                                                    (size_t)kLogitsScratchBytes);
        const size_t logits = ring + (size_t)8 * p.out_rows;
        work = std::max({attention, logits, (size_t)4 * p.kpd * sizeof(WT)});
    } else {
        // A fused cross query's tile sits past the cross attention's own
        // area, and a cooperative join's partials after it.
        work = std::max({product + kCrossQueryOffset, attention,
                         (size_t)kCrossQueryOffset + sizeof(float) * kMaxCrossSplits * 66});
    }
    return (work + 127) / 128 * 128;
}

template <typename WT, int NT>
size_t shared_bytes(const StepParams& p, int max_chunk) {
    return 1024 + (size_t)p.stages * p.stage_bytes + 16 * kMaxStages + work_bytes<WT, NT>(p, max_chunk);
}

template <typename WT, int NT>
void launch_typed(const StepParams& p, int max_chunk, int grid, cudaStream_t stream) {
    const size_t smem = shared_bytes<WT, NT>(p, max_chunk);
    auto kernel = p.umma ? decode_kernel<WT, NT, true> : decode_kernel<WT, NT, false>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) throw std::runtime_error(std::string("decode kernel shared memory: ") + cudaGetErrorString(e));
    StepParams copy = p;
    void* args[] = {&copy};
    e = cudaLaunchCooperativeKernel((const void*)kernel, grid, kBlockThreads, args, smem, stream);
    if (e != cudaSuccess) throw std::runtime_error(std::string("decode kernel launch: ") + cudaGetErrorString(e));
}

template <typename WT, int NT>
int occupancy_typed(const StepParams& p, int max_chunk) {
    const size_t smem = shared_bytes<WT, NT>(p, max_chunk);
    auto kernel = p.umma ? decode_kernel<WT, NT, true> : decode_kernel<WT, NT, false>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, kBlockThreads, smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return blocks;
}

// Input rows per tile: 8, 16, or 32 (more rows run as several tiles); the
// host may ask for fewer (p.tile_columns) when the tile's two planes leave
// too little shared memory for the weight stream.
inline int tile_columns(const StepParams& p) {
    const int rows = std::max(p.rows, p.out_rows);
    const int wanted = rows <= 8 ? 1 : (rows <= 16 ? 2 : 4);
    return p.tile_columns > 0 && p.tile_columns < wanted ? p.tile_columns : wanted;
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

template <typename WT>
size_t work_rows(const StepParams& p, int max_chunk) {
    switch (tile_columns(p)) {
    case 1: return work_bytes<WT, 1>(p, max_chunk);
    case 2: return work_bytes<WT, 2>(p, max_chunk);
    default: return work_bytes<WT, 4>(p, max_chunk);
    }
}

}  // namespace

int decode_tile_rows(const StepParams& p) { return 8 * tile_columns(p); }

size_t decode_work_bytes(bool half, const StepParams& p, int max_chunk) {
    return (half ? work_rows<__half>(p, max_chunk) : work_rows<__nv_bfloat16>(p, max_chunk)) + 16 * kMaxStages +
           1024;
}

int decode_blocks_per_sm(bool half, const StepParams& p, int max_chunk) {
    return half ? occupancy_rows<__half>(p, max_chunk) : occupancy_rows<__nv_bfloat16>(p, max_chunk);
}

void launch_decode(bool half, const StepParams& p, int max_chunk, int grid, cudaStream_t stream) {
    if (p.width > 32 * kNormMaxPerLane) throw std::invalid_argument("widths above 1536 are not supported");
    if (p.head_width > 64) throw std::invalid_argument("heads wider than 64 are not supported");
    if (p.stages < 1 || p.stages > kMaxStages || p.stage_bytes % 1024 != 0)
        throw std::invalid_argument("weight stream stages out of range");
    if (half) launch_rows<__half>(p, max_chunk, grid, stream);
    else launch_rows<__nv_bfloat16>(p, max_chunk, grid, stream);
}

}  // namespace wsp
