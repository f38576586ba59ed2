// The decoder token loop's kernels for sm_100a.
//
// Reference semantics (paths within eyalamirmusic/WhisperEACP):
//   embed            Lib/WhisperEACP/Kernels/Embed.h:38-64
//   layer norm       Lib/WhisperEACP/Kernels/LayerNorm.h:19-98 (two-pass, eps 1e-5)
//   projections      Lib/WhisperEACP/Kernels/Linear.h:128-276 (bias, exact GELU, residual)
//   attention        Lib/WhisperEACP/Kernels/SingleQueryAttention.h:62-373,397-501,
//                    Attention.h:75-209 (scale on the scores, causal mask for the prompt)
//   masked argmax    Lib/WhisperEACP/Kernels/Argmax.h:83-201, Argmax.cpp:47-80
#include "common.cuh"
#include "kernels.cuh"

#include <algorithm>
#include <stdexcept>

namespace wsp {

namespace {

template <Storage S> struct StorageType;
template <> struct StorageType<Storage::f16> { using type = __half; };
template <> struct StorageType<Storage::bf16> { using type = __nv_bfloat16; };

// ------------------------------------------------------------------ embed

// h[r, :] = token_table[ring[b, position+t]] + position_table[position+t]
template <typename WT>
__global__ void __launch_bounds__(kThreads) embed_kernel(EmbedArgs a) {
    const int r = blockIdx.x;
    if (r >= a.rows) return;
    const int b = r / a.tokens, t = r % a.tokens;
    const int p = *a.position + t;
    uint32_t token = a.ring[(size_t)b * a.ring_stride + p];
    if (token >= (uint32_t)a.vocabulary) {
        if (threadIdx.x == 0) atomicOr(a.error, 1);
        token = 0;
    }
    const WT* row = static_cast<const WT*>(a.token_table) + (size_t)token * a.token_stride;
    const float* pos = a.position_table + (size_t)p * a.width;
    float* out = a.hidden + (size_t)r * a.width;
    for (int c = threadIdx.x; c < a.width; c += kThreads)
        out[c] = Half16<WT>::to_float(row[c]) + pos[c];
}

// ------------------------------------------------------------- layer norm

constexpr int kNormMaxPerLane = 48;  // widths up to 1536

// One warp per row, the row held in registers: mean, then the centred
// variance, then (x - mean) * rsqrt(var + eps) * gamma + beta.
template <typename WT>
__global__ void __launch_bounds__(kThreads) layer_norm_kernel(LayerNormArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * kWarps + warp;
    if (r >= a.rows) return;
    const float* x = a.input + ((size_t)r * a.row_step + a.row_offset) * a.width;
    float v[kNormMaxPerLane];
    float total = 0.f;
#pragma unroll
    for (int i = 0; i < kNormMaxPerLane; ++i) {
        const int c = lane + 32 * i;
        v[i] = c < a.width ? x[c] : 0.f;
        total += v[i];
    }
    const float mean = warp_sum(total) / (float)a.width;
    float centred = 0.f;
#pragma unroll
    for (int i = 0; i < kNormMaxPerLane; ++i) {
        const int c = lane + 32 * i;
        const float dv = c < a.width ? v[i] - mean : 0.f;
        centred += dv * dv;
    }
    const float variance = warp_sum(centred) / (float)a.width;
    const float scale = rsqrtf(variance + 1e-5f);
    WT* out = static_cast<WT*>(a.output) + (size_t)r * a.ld_output;
#pragma unroll
    for (int i = 0; i < kNormMaxPerLane; ++i) {
        const int c = lane + 32 * i;
        if (c < a.width) {
            const float y = (v[i] - mean) * scale * a.gamma[c] + a.beta[c];
            out[c] = Half16<WT>::from_float(y);
            if (a.hidden_copy) a.hidden_copy[(size_t)r * a.width + c] = y;
        }
    }
}

// --------------------------------------------------------------- products

// Y[r, n] = sum_k X[r, k] W[n, k]: the weight rows are the MMA's M side and the
// activation rows its N side (swap-AB), so one m16n8k16 covers 16 weight rows
// against 8 rows of activations.  A CTA owns 16 weight rows and RT = 8*NT
// activation rows; its 8 warps split K in 32-wide chunks and are folded in
// shared memory in a fixed order, so the sums are deterministic.
//
// Within a 32-wide chunk, lane (g, t) loads 16 bytes of weight row g and of
// row g+8, and 16 bytes of each activation row, all at k = 8t..8t+7.  The
// two MMA k-steps take the lower and upper halves; since the activation
// fragments are loaded under the same k permutation as the weight fragments,
// each product pairs the right elements, and no ldmatrix or shared staging is
// needed to stream the weights with full 16-byte loads.
template <int NT> struct GemmDepth { static constexpr int value = NT <= 2 ? 4 : (NT <= 4 ? 2 : 1); };

template <typename WT, int NT, Epilogue EPI>
__global__ void __launch_bounds__(kThreads, 2) gemm_kernel(GemmArgs a) {
    constexpr int RT = 8 * NT;
    constexpr int U = GemmDepth<NT>::value;
    extern __shared__ float smem[];
    float* red = smem;                    // [8][16][RT]
    float* tile = smem + kWarps * 16 * RT;  // [16][RT] (logits)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;
    const int n_tiles = (a.n + 15) / 16;
    const int r_tiles = (a.rows + RT - 1) / RT;
    const int chunks = a.kp / 32;
    const WT* W = static_cast<const WT*>(a.weight);
    const WT* X = static_cast<const WT*>(a.input);
    int position = 0;
    if constexpr (EPI == Epilogue::qkv) position = *a.position;

    for (int item = blockIdx.x; item < n_tiles * r_tiles; item += gridDim.x) {
        const int n_tile = item / r_tiles, r_tile = item % r_tiles;
        const int n0 = n_tile * 16, r0 = r_tile * RT;
        float acc[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

        const WT* w_lo = W + (size_t)min(n0 + gq, a.n - 1) * a.kp + 8 * tq;
        const WT* w_hi = W + (size_t)min(n0 + gq + 8, a.n - 1) * a.kp + 8 * tq;
        const WT* x_row[NT];
        bool x_ok[NT];
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            const int r = r0 + 8 * j + gq;
            x_ok[j] = r < a.rows;
            x_row[j] = X + (size_t)(x_ok[j] ? r : 0) * a.kp + 8 * tq;
        }

        for (int base = warp; base < chunks; base += kWarps * U) {
            uint4 A[U][2];
            uint4 B[U][NT];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = base + kWarps * u;
                if (c < chunks) {
                    A[u][0] = load_stream(w_lo + c * 32);
                    A[u][1] = load_stream(w_hi + c * 32);
#pragma unroll
                    for (int j = 0; j < NT; ++j)
                        B[u][j] = x_ok[j] ? load_cached(x_row[j] + c * 32) : make_uint4(0, 0, 0, 0);
                } else {
                    A[u][0] = A[u][1] = make_uint4(0, 0, 0, 0);
#pragma unroll
                    for (int j = 0; j < NT; ++j) B[u][j] = make_uint4(0, 0, 0, 0);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t a0[4] = {A[u][0].x, A[u][1].x, A[u][0].y, A[u][1].y};
                const uint32_t a1[4] = {A[u][0].z, A[u][1].z, A[u][0].w, A[u][1].w};
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const uint32_t b0[2] = {B[u][j].x, B[u][j].y};
                    const uint32_t b1[2] = {B[u][j].z, B[u][j].w};
                    mma_16816<WT>(acc[j], a0, b0);
                    mma_16816<WT>(acc[j], a1, b1);
                }
            }
        }

        // Fold the eight warps' K slices.
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            const int col = 8 * j + 2 * tq;
            red[(warp * 16 + gq) * RT + col] = acc[j][0];
            red[(warp * 16 + gq) * RT + col + 1] = acc[j][1];
            red[(warp * 16 + gq + 8) * RT + col] = acc[j][2];
            red[(warp * 16 + gq + 8) * RT + col + 1] = acc[j][3];
        }
        __syncthreads();
        for (int o = threadIdx.x; o < 16 * RT; o += kThreads) {
            const int nl = o / RT, rl = o % RT;
            const int n = n0 + nl, r = r0 + rl;
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) v += red[(w * 16 + nl) * RT + rl];
            const bool live = n < a.n && r < a.rows;
            if (live && a.bias) v += a.bias[n];
            if constexpr (EPI == Epilogue::store) {
                if (live) a.out[(size_t)r * a.ld_out + n] = v;
            } else if constexpr (EPI == Epilogue::residual) {
                if (live) a.out[(size_t)r * a.ld_out + n] += v;
            } else if constexpr (EPI == Epilogue::gelu) {
                if (live) static_cast<WT*>(a.out16)[(size_t)r * a.ld_out16 + n] = Half16<WT>::from_float(gelu_exact(v));
            } else if constexpr (EPI == Epilogue::qkv) {
                if (live) {
                    if (n < a.width) {
                        a.out[(size_t)r * a.ld_out + n] = v;
                    } else {
                        const int which = (n - a.width) / a.width;
                        const int c = (n - a.width) - which * a.width;
                        const int b = r / a.tokens, t = r % a.tokens;
                        WT* cache = static_cast<WT*>(which == 0 ? a.self_keys : a.self_values);
                        cache[((size_t)b * a.max_positions + position + t) * a.width + c] = Half16<WT>::from_float(v);
                    }
                }
            } else if constexpr (EPI == Epilogue::logits) {
                if (live && a.logits) a.logits[(size_t)r * a.ld_logits + n] = v;
                tile[nl * RT + rl] = v;
            }
        }
        if constexpr (EPI == Epilogue::logits) {
            __syncthreads();
            // The tile's candidate for each row, scanned in ascending column
            // order keeping the first maximum (Argmax.h:93-110).
            for (int rl = threadIdx.x; rl < RT; rl += kThreads) {
                const int r = r0 + rl;
                if (r >= a.rows) continue;
                float best_v = -INFINITY;
                uint32_t best_i = kUnchosen;
                for (int nl = 0; nl < 16; ++nl) {
                    const int n = n0 + nl;
                    if (n >= a.n) break;
                    if (a.mask && a.mask[n] != 0.f) continue;
                    const float v = tile[nl * RT + rl];
                    if (best_i == kUnchosen || v > best_v) { best_v = v; best_i = (uint32_t)n; }
                }
                a.candidate_values[(size_t)r * n_tiles + n_tile] = best_v;
                a.candidate_indices[(size_t)r * n_tiles + n_tile] = best_i;
            }
        }
        __syncthreads();
    }
}

// -------------------------------------------------------------- attention

constexpr int kMaxChunk = 2048;
constexpr int kMaxHeadWidth = 64;

// One CTA per (row, head, split): scores of this split's keys, their maximum,
// the exponentials and their sum, and the unnormalised weighted value row --
// the partial a split-softmax joins exactly (SingleQueryAttention.h:11-37).
template <typename WT>
__global__ void __launch_bounds__(kThreads) attention_partial_kernel(AttentionArgs a) {
    __shared__ float q[kMaxHeadWidth];
    __shared__ float scores[kMaxChunk];
    __shared__ float scratch[kWarps];
    __shared__ float fold[kThreads];

    const int split = blockIdx.x % a.splits;
    const int head = (blockIdx.x / a.splits) % a.heads;
    const int r = blockIdx.x / (a.splits * a.heads);
    const int D = a.head_width;
    const int b = r / a.tokens, t = r % a.tokens;
    const int keys = a.causal ? (*a.position + t + 1) : a.key_count;
    const int k0 = split * a.chunk;
    const int k1 = min(keys, k0 + a.chunk);
    float* out = a.partial + (((size_t)r * a.heads + head) * a.splits + split) * (D + 2);

    if (k0 >= k1) {
        for (int c = threadIdx.x; c < D + 2; c += kThreads) out[c] = c == 0 ? -INFINITY : 0.f;
        return;
    }
    for (int c = threadIdx.x; c < D; c += kThreads)
        q[c] = a.queries[(size_t)r * a.ld_queries + head * D + c] * a.scale;
    __syncthreads();

    const WT* K = static_cast<const WT*>(a.keys) + (size_t)b * a.window_stride + (size_t)head * D;
    const WT* V = static_cast<const WT*>(a.values) + (size_t)b * a.window_stride + (size_t)head * D;
    const int n = k1 - k0;

    float local_max = -INFINITY;
    for (int j = threadIdx.x; j < n; j += kThreads) {
        const WT* krow = K + (size_t)(k0 + j) * a.key_stride;
        float s = 0.f;
        if (D % 8 == 0) {
            for (int c = 0; c < D; c += 8) {
                const uint4 u = load_cached(krow + c);
                const float2 f0 = Half16<WT>::pair_to_float2(u.x), f1 = Half16<WT>::pair_to_float2(u.y);
                const float2 f2 = Half16<WT>::pair_to_float2(u.z), f3 = Half16<WT>::pair_to_float2(u.w);
                s += q[c] * f0.x + q[c + 1] * f0.y + q[c + 2] * f1.x + q[c + 3] * f1.y +
                     q[c + 4] * f2.x + q[c + 5] * f2.y + q[c + 6] * f3.x + q[c + 7] * f3.y;
            }
        } else {
            for (int c = 0; c < D; ++c) s += q[c] * Half16<WT>::to_float(krow[c]);
        }
        scores[j] = s;
        local_max = fmaxf(local_max, s);
    }
    const float m = block_max(local_max, scratch);
    float local_sum = 0.f;
    for (int j = threadIdx.x; j < n; j += kThreads) {
        const float p = __expf(scores[j] - m);
        scores[j] = p;
        local_sum += p;
    }
    const float l = block_sum(local_sum, scratch);  // contains a __syncthreads

    // Weighted values: thread (group, channel) walks the keys of its group.
    const int groups = kThreads / D;
    const int c = threadIdx.x % D, g = threadIdx.x / D;
    float acc = 0.f;
    if (g < groups)
        for (int j = g; j < n; j += groups)
            acc += scores[j] * Half16<WT>::to_float(V[(size_t)(k0 + j) * a.key_stride + c]);
    fold[threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.x < D) {
        float o = 0.f;
        for (int gg = 0; gg < groups; ++gg) o += fold[gg * D + threadIdx.x];
        out[2 + threadIdx.x] = o;
    }
    if (threadIdx.x == 0) {
        out[0] = m;
        out[1] = l;
    }
}

// Joins the splits of each (row, head): rescale by exp(m_s - m), sum, divide.
template <typename WT>
__global__ void __launch_bounds__(kThreads) attention_combine_kernel(CombineArgs a) {
    const int r = blockIdx.x;
    const int D = a.head_width;
    const int width = a.heads * D;
    WT* out = static_cast<WT*>(a.output) + (size_t)r * a.ld_output;
    for (int at = threadIdx.x; at < width; at += kThreads) {
        const int head = at / D, c = at % D;
        const float* p = a.partial + ((size_t)r * a.heads + head) * a.splits * (D + 2);
        float m = -INFINITY;
        for (int s = 0; s < a.splits; ++s) m = fmaxf(m, p[s * (D + 2)]);
        float l = 0.f, o = 0.f;
        for (int s = 0; s < a.splits; ++s) {
            const float ms = p[s * (D + 2)];
            if (ms == -INFINITY) continue;
            const float f = __expf(ms - m);
            l += p[s * (D + 2) + 1] * f;
            o += p[s * (D + 2) + 2 + c] * f;
        }
        float y = o / l;
        if (a.bias) y += a.bias[at];
        out[at] = Half16<WT>::from_float(y);
    }
}

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

__global__ void advance_position_kernel(int* position, int tokens) { *position += tokens; }

template <typename WT>
__global__ void to_storage_kernel(const float* in, WT* out, long long count) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (long long)gridDim.x * blockDim.x)
        out[i] = Half16<WT>::from_float(in[i]);
}

template <typename WT, int NT, Epilogue EPI>
void gemm_launch_one(const GemmArgs& a, int sm_count, cudaStream_t stream) {
    constexpr int RT = 8 * NT;
    const int items = gemm_column_tiles(a.n) * ((a.rows + RT - 1) / RT);
    // At most 36 KB (RT = 64), under the 48 KB a launch may ask for without an opt-in.
    const size_t smem = sizeof(float) * (kWarps * 16 * RT + 16 * RT);
    const int grid = std::max(1, std::min(items, sm_count * 2));
    gemm_kernel<WT, NT, EPI><<<grid, kThreads, smem, stream>>>(a);
}

template <typename WT, Epilogue EPI>
void gemm_launch_rows(const GemmArgs& a, int sm_count, cudaStream_t stream) {
    if (a.rows <= 8) gemm_launch_one<WT, 1, EPI>(a, sm_count, stream);
    else if (a.rows <= 16) gemm_launch_one<WT, 2, EPI>(a, sm_count, stream);
    else if (a.rows <= 32) gemm_launch_one<WT, 4, EPI>(a, sm_count, stream);
    else gemm_launch_one<WT, 8, EPI>(a, sm_count, stream);
}

template <typename WT>
void gemm_dispatch(Epilogue e, const GemmArgs& a, int sm_count, cudaStream_t stream) {
    switch (e) {
    case Epilogue::qkv: gemm_launch_rows<WT, Epilogue::qkv>(a, sm_count, stream); break;
    case Epilogue::store: gemm_launch_rows<WT, Epilogue::store>(a, sm_count, stream); break;
    case Epilogue::residual: gemm_launch_rows<WT, Epilogue::residual>(a, sm_count, stream); break;
    case Epilogue::gelu: gemm_launch_rows<WT, Epilogue::gelu>(a, sm_count, stream); break;
    case Epilogue::logits: gemm_launch_rows<WT, Epilogue::logits>(a, sm_count, stream); break;
    }
}

}  // namespace

int gemm_column_tiles(int n) { return (n + 15) / 16; }

void launch_embed(Storage s, const EmbedArgs& a, cudaStream_t stream) {
    if (s == Storage::f16) embed_kernel<__half><<<a.rows, kThreads, 0, stream>>>(a);
    else embed_kernel<__nv_bfloat16><<<a.rows, kThreads, 0, stream>>>(a);
}

void launch_layer_norm(Storage s, const LayerNormArgs& a, cudaStream_t stream) {
    if (a.width > 32 * kNormMaxPerLane) throw std::invalid_argument("layer norm width above 1536");
    const int grid = (a.rows + kWarps - 1) / kWarps;
    if (s == Storage::f16) layer_norm_kernel<__half><<<grid, kThreads, 0, stream>>>(a);
    else layer_norm_kernel<__nv_bfloat16><<<grid, kThreads, 0, stream>>>(a);
}

void launch_gemm(Storage s, Epilogue e, const GemmArgs& a, int sm_count, cudaStream_t stream) {
    if (a.kp % 32 != 0) throw std::invalid_argument("product inner extent must be padded to 32");
    if (s == Storage::f16) gemm_dispatch<__half>(e, a, sm_count, stream);
    else gemm_dispatch<__nv_bfloat16>(e, a, sm_count, stream);
}

void launch_attention_partial(Storage s, const AttentionArgs& a, cudaStream_t stream) {
    if (a.head_width > kMaxHeadWidth || a.chunk > kMaxChunk)
        throw std::invalid_argument("attention head width above 64 or key chunk above 2048");
    const int grid = a.rows * a.heads * a.splits;
    if (s == Storage::f16) attention_partial_kernel<__half><<<grid, kThreads, 0, stream>>>(a);
    else attention_partial_kernel<__nv_bfloat16><<<grid, kThreads, 0, stream>>>(a);
}

void launch_attention_combine(Storage s, const CombineArgs& a, cudaStream_t stream) {
    if (s == Storage::f16) attention_combine_kernel<__half><<<a.rows, kThreads, 0, stream>>>(a);
    else attention_combine_kernel<__nv_bfloat16><<<a.rows, kThreads, 0, stream>>>(a);
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

void launch_advance_position(int* position, int tokens, cudaStream_t stream) {
    advance_position_kernel<<<1, 1, 0, stream>>>(position, tokens);
}

void launch_to_storage(Storage s, const float* in, void* out, long long count, cudaStream_t stream) {
    const int grid = (int)std::min<long long>((count + kThreads - 1) / kThreads, 148LL * 16);
    if (s == Storage::f16) to_storage_kernel<__half><<<grid, kThreads, 0, stream>>>(in, static_cast<__half*>(out), count);
    else to_storage_kernel<__nv_bfloat16><<<grid, kThreads, 0, stream>>>(in, static_cast<__nv_bfloat16*>(out), count);
}

}  // namespace wsp
