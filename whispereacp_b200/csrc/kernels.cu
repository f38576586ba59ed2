// Kernels outside the decode step (sm_100a): the standalone masked argmax of
// Argmax.h:83-201 / Argmax.cpp:47-80 (WhisperEACP, Lib/WhisperEACP/Kernels).
#include "common.cuh"
#include "kernels.cuh"

#include <algorithm>
#include <mutex>
#include <stdexcept>

namespace wsp {

namespace {

// ----------------------------------------------------------------- argmax

__device__ void block_fold_candidate(float& v, uint32_t& i) {
    __shared__ float sv[kThreads];
    __shared__ uint32_t si[kThreads];
    sv[threadIdx.x] = v;
    si[threadIdx.x] = i;
    __syncthreads();
    for (int stride = kThreads / 2; stride > 0; stride >>= 1) {
        if (threadIdx.x < stride) {
            const float ov = sv[threadIdx.x + stride];
            const uint32_t oi = si[threadIdx.x + stride];
            if (candidate_better(ov, oi, sv[threadIdx.x], si[threadIdx.x])) {
                sv[threadIdx.x] = ov;
                si[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    v = sv[0];
    i = si[0];
}

__global__ void __launch_bounds__(kThreads) argmax_final_kernel(ArgmaxFinalArgs a) {
    const int r = blockIdx.x;
    const float* values = a.candidate_values + (size_t)r * a.candidates;
    const uint32_t* indices = a.candidate_indices + (size_t)r * a.candidates;
    float bv = -INFINITY;
    uint32_t bi = kUnchosen;
    for (int c = threadIdx.x; c < a.candidates; c += kThreads)
        if (candidate_better(values[c], indices[c], bv, bi)) { bv = values[c]; bi = indices[c]; }
    block_fold_candidate(bv, bi);
    if (threadIdx.x == 0) {
        const uint32_t chosen = bi == kUnchosen ? 0u : bi;  // Argmax.h:190-193
        if (a.row_tokens) a.row_tokens[r] = chosen;
        const int b = r / a.rows_per_window, t = r % a.rows_per_window;
        if (a.ring && t == a.rows_per_window - 1)
            a.ring[(size_t)b * a.ring_stride + *a.position + a.step_tokens] = chosen;
    }
}

// ArgmaxPartial (Argmax.h:83-141): group `part` of a row scans its strided
// share in ascending order and keeps the first maximum it meets.
__global__ void __launch_bounds__(kThreads) argmax_partial_kernel(const float* logits, const float* mask,
                                                                  int length, int groups_per_row,
                                                                  float* cv, uint32_t* ci) {
    const int row = blockIdx.x / groups_per_row, part = blockIdx.x % groups_per_row;
    const float* base = logits + (size_t)row * length;
    float bv = -INFINITY;
    uint32_t bi = kUnchosen;
    for (int j = part * kThreads + threadIdx.x; j < length; j += groups_per_row * kThreads) {
        if (mask && mask[j] != 0.f) continue;
        const float v = base[j];
        if (bi == kUnchosen || v > bv) { bv = v; bi = (uint32_t)j; }
    }
    block_fold_candidate(bv, bi);
    if (threadIdx.x == 0) {
        cv[blockIdx.x] = bv;
        ci[blockIdx.x] = bi;
    }
}

}  // namespace

// The no-allocation argmax's scratch: 65536 candidate pairs (512 KB), values
// first.  It is part of the module's static device memory, loaded with the
// library, so a call that uses it allocates nothing.  Nothing in it has to
// start at zero: the partial pass writes every slot the final pass reads.
static __device__ __align__(256) unsigned char no_alloc_scratch[kNoAllocArgmaxCandidates * 8];

cudaError_t no_alloc_argmax_scratch(int device, void** scratch) {
    constexpr int kMaxDevices = 64;
    static std::mutex lock;
    static void* addresses[kMaxDevices] = {};
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> guard(lock);
    if (addresses[device] == nullptr) {
        void* address = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&address, no_alloc_scratch);
        if (e != cudaSuccess) return e;
        addresses[device] = address;
    }
    *scratch = addresses[device];
    return cudaSuccess;
}

void launch_argmax_final(const ArgmaxFinalArgs& a, cudaStream_t stream) {
    argmax_final_kernel<<<a.rows, kThreads, 0, stream>>>(a);
}

int argmax_groups_per_row(int length) {
    const int per_group = kThreads * 8;  // about eight elements a thread (Argmax.cpp:17-24)
    return std::max(1, (length + per_group - 1) / per_group);
}

void launch_argmax_rows(const float* logits, const float* mask, uint32_t* out, int rows, int length,
                        float* cv, uint32_t* ci, int groups_per_row, cudaStream_t stream) {
    argmax_partial_kernel<<<rows * groups_per_row, kThreads, 0, stream>>>(logits, mask, length,
                                                                         groups_per_row, cv, ci);
    ArgmaxFinalArgs f{};
    f.candidate_values = cv;
    f.candidate_indices = ci;
    f.candidates = groups_per_row;
    f.rows = rows;
    f.rows_per_window = 1;
    f.step_tokens = 1;
    f.row_tokens = out;
    argmax_final_kernel<<<rows, kThreads, 0, stream>>>(f);
}

}  // namespace wsp
