// The weight-stream schedule of a decode-kernel launch: for every CTA, the
// units of weights it streams through its shared-memory ring in one step, in
// the order its ops consume them.  Built on the host once per op list; the
// kernel's thread 0 only walks it.
#pragma once

#include "step.cuh"

#include <algorithm>
#include <utility>
#include <vector>

namespace wsp {

// A run of `tiles` contiguous 16-row tiles of `chunks` 1 KB chunks.  A stream
// unit is `group` whole tiles, or -- for a tile larger than a stage -- a
// k-block of one tile.
struct Region {
    const unsigned char* base;
    int tiles, chunks, group;
};

inline int schedule_row_tiles(int rows, int rt) { return (rows + rt - 1) / rt; }
inline int schedule_round16(int n) { return (n + 15) / 16 * 16; }

// Items of an op; CTA c takes items c, c + grid, ...  rt: input rows of a
// product's tile (8 * NT of the launch).
inline int op_items(const StepParams& p, const StepOp& op, int rt) {
    switch (op.kind) {
    case kOpProduct: return ((op.n + 15) / 16) * schedule_row_tiles(p.rows, rt) * (op.kparts > 1 ? op.kparts : 1);
    case kOpLogits: return ((p.vocabulary + 15) / 16) * schedule_row_tiles(p.out_rows, rt);
    }
    return 0;
}

// Weight region `region` of item `item` of an op; false when there is none.
inline bool item_region(const StepParams& p, const StepOp& op, int item, int region, int rt, Region& out) {
    switch (op.kind) {
    case kOpProduct:
    case kOpLogits: {
        if (region != 0) return false;
        const int n = op.kind == kOpProduct ? op.n : p.vocabulary;
        const int kp = op.kind == kOpProduct ? op.kp : p.kpd;
        const void* w = op.kind == kOpProduct ? op.weight : p.token_table;
        const int n_tiles = (n + 15) / 16, tile = item % n_tiles;
        // A split product's item: part item / (tiles x row tiles), its share
        // of the tile's chunks (contiguous in the fragment-packed layout).
        const int parts = op.kind == kOpProduct && op.kparts > 1 ? op.kparts : 1;
        const int part = item / (n_tiles * schedule_row_tiles(p.rows, rt));
        const int chunks = kp / 32 / parts;
        out = Region{static_cast<const unsigned char*>(w) + ((size_t)tile * (kp / 32) + (size_t)part * chunks) * 1024,
                     1, chunks, 1};
        return true;
    }
    }
    return false;
}

// Appends the units of a region: whole-tile groups, or k-blocks of a tile
// larger than a stage.
inline void append_region(const Region& r, int stage_chunks, std::vector<ScheduleEntry>& out) {
    if (r.chunks > stage_chunks) {
        const int blocks = (r.chunks + stage_chunks - 1) / stage_chunks;
        for (int t = 0; t < r.tiles; ++t)
            for (int b = 0; b < blocks; ++b) {
                const unsigned bytes = (unsigned)std::min(stage_chunks, r.chunks - b * stage_chunks) * 1024u;
                out.push_back(schedule_entry(r.base + ((size_t)t * r.chunks + (size_t)b * stage_chunks) * 1024, bytes));
            }
        return;
    }
    for (int t0 = 0; t0 < r.tiles; t0 += r.group) {
        const unsigned bytes = (unsigned)(std::min(r.group, r.tiles - t0) * r.chunks) * 1024u;
        out.push_back(schedule_entry(r.base + (size_t)t0 * r.chunks * 1024, bytes));
    }
}

// Cross attention: the CTA's items (cta, cta + grid, ...), each item's
// units (one per `chunk` keys) in order, as op_cross_attention reads them;
// with a fused query, the head's q weight tiles before them.
inline void append_cross_units(const StepParams& p, const StepOp& op, int cta, int grid, int stage_chunks,
                               std::vector<ScheduleEntry>& out) {
    const int S = op.splits, H = p.heads;
    const int items = p.rows * H * S;
    const int units = (op.key_count + op.chunk - 1) / op.chunk;
    const size_t key_bytes = 4 * (size_t)p.head_width;
    for (int it = cta; it < items; it += grid) {
        const int split = it % S, head = (it / S) % H, r = it / (S * H), b = r / p.tokens;
        const int count = std::max(0, std::min(op.span, units - split * op.span));
        if (op.weight) {
            // A fused query: the head's 16-row q tiles first (cross_query).
            const int head_tiles = schedule_round16(p.head_width) / 16;
            append_region(Region{static_cast<const unsigned char*>(op.weight) +
                                     (size_t)head * head_tiles * (op.kp / 32) * 1024,
                                 head_tiles, op.kp / 32, 1},
                          stage_chunks, out);
        }
        for (int t = 0; t < count; ++t) {
            const int k0 = (split * op.span + t) * op.chunk;
            const int n = std::min(op.chunk, op.key_count - k0);
            const size_t element = (size_t)b * op.window_stride + (size_t)head * op.head_stride +
                                   (size_t)k0 * op.key_stride;
            out.push_back(schedule_entry(static_cast<const unsigned char*>(op.keys) + element * 2,
                                         (unsigned)(n * key_bytes)));
        }
    }
}

// Tensor-core product: item (m tile of 128 weight rows, group of umma_rows
// rows, K split), CTA c taking items c, c + grid, ...; the split's weight
// blocks (16 KB per 64 columns), umma_blocks to a unit, as product_umma
// reads them.
// (The rows' activations come through the product's own ring.)
inline int umma_items(const StepParams& p, const StepOp& op) {
    return ((op.n + 127) / 128) * ((p.rows + p.umma_rows - 1) / p.umma_rows) * (op.ksplit > 1 ? op.ksplit : 1);
}
inline void append_umma_units(const StepParams& p, const StepOp& op, int cta, int grid,
                              std::vector<ScheduleEntry>& out) {
    const int kblocks = op.kp / 64;
    for (int item = cta; item < umma_items(p, op); item += grid) {
        const UmmaItem u = umma_item(p, op, item);
        for (int kb = u.kb0; kb < u.kb1; kb += p.umma_blocks) {
            const int n = std::min(p.umma_blocks, u.kb1 - kb);
            out.push_back(schedule_entry(static_cast<const unsigned char*>(op.weight) + ((size_t)u.m * kblocks + kb) * 16384,
                                         16384u * (unsigned)n));
        }
    }
}

// Tensor-core logits: item (128 vocabulary rows, 128 sampled rows), CTA c
// taking items c, c + grid, ...; the token table's k-blocks of the item's
// vocabulary tile, umma_blocks to a unit, as logits_umma reads them.
inline void append_logits_umma_units(const StepParams& p, int cta, int grid, std::vector<ScheduleEntry>& out) {
    const int kblocks = p.kpd / 64, vocab_tiles = (p.vocabulary + 127) / 128;
    const int items = vocab_tiles * ((p.out_rows + 127) / 128);
    for (int item = cta; item < items; item += grid) {
        const int m = item % vocab_tiles;
        for (int kb = 0; kb < kblocks; kb += p.umma_blocks) {
            const int n = std::min(p.umma_blocks, kblocks - kb);
            out.push_back(schedule_entry(static_cast<const unsigned char*>(p.token_table) +
                                             ((size_t)m * kblocks + kb) * 16384,
                                         16384u * (unsigned)n));
        }
    }
}

// What an op reads straight from memory that no op writes, for the
// producers to prefetch into L2 just ahead of it: LayerNorm gains and
// offsets, biases, the mask, a fused out-projection's head columns (2 KB of
// every 16-row tile).
inline void op_prefetches(const StepParams& p, const StepOp& op,
                          std::vector<std::pair<const void*, unsigned long long>>& out) {
    const unsigned long long row = (unsigned long long)p.width * 4;
    auto add = [&](const void* ptr, unsigned long long bytes) {
        if (ptr && bytes) out.push_back({ptr, bytes});
    };
    switch (op.kind) {
    case kOpProduct:
        add(op.gamma, row);
        add(op.beta, row);
        add(op.bias, 4ull * op.n);
        add(op.addend_bias, row);
        break;
    case kOpNorm:
        add(op.gamma, row);
        add(op.beta, row);
        break;
    case kOpLogits:
        add(p.final_gamma, row);
        add(p.final_beta, row);
        if (p.mask)
            for (unsigned long long o = 0, all = 4ull * p.vocabulary; o < all; o += 4096)
                add(reinterpret_cast<const unsigned char*>(p.mask) + o, std::min(4096ull, all - o));
        break;
    case kOpCrossAttention:
        add(op.value_bias, row);
        add(op.gamma, row);
        add(op.beta, row);
        add(op.bias, 4ull * op.n);
        add(op.addend_bias, row);
        break;
    }
    if (op.out_weight) {
        const int chunks = p.kpd / 32, tiles = (p.width + 15) / 16;
        for (int h = 0; h < p.heads; ++h)
            for (int t = 0; t < tiles; ++t)
                add(static_cast<const unsigned char*>(op.out_weight) + ((size_t)t * chunks + 2 * h) * 1024, 2048);
    }
}

// The per-CTA schedules of a launch, concatenated, and their offsets.  Ahead
// of each op's units, a CTA's schedule carries its share of that op's
// prefetches (entry j of op k goes to CTA (j + 7k) mod grid).
inline void build_schedule(const StepParams& p, const std::vector<StepOp>& ops, int grid, int rt,
                           std::vector<ScheduleEntry>& units, std::vector<unsigned>& offsets) {
    const int stage_chunks = p.stage_bytes / 1024;
    units.clear();
    offsets.assign(1, 0u);
    std::vector<std::vector<std::pair<const void*, unsigned long long>>> prefetches(ops.size());
    for (size_t k = 0; k < ops.size(); ++k) op_prefetches(p, ops[k], prefetches[k]);
    for (int cta = 0; cta < grid; ++cta) {
        for (size_t k = 0; k < ops.size(); ++k) {
            const StepOp& op = ops[k];
            const auto& pf = prefetches[k];
            for (size_t j = (size_t)((cta - (long long)(7 * k) % grid + grid) % grid); j < pf.size(); j += grid)
                units.push_back(ScheduleEntry{(unsigned long long)(size_t)pf[j].first, pf[j].second | kPrefetchOnly});
            if (op.kind == kOpCrossAttention) {
                append_cross_units(p, op, cta, grid, stage_chunks, units);
                continue;
            }
            if (op.kind == kOpProduct && p.umma) {
                append_umma_units(p, op, cta, grid, units);
                continue;
            }
            if (op.kind == kOpLogits && p.umma) {
                append_logits_umma_units(p, cta, grid, units);
                continue;
            }
            const int items = op_items(p, op, rt);
            for (int item = cta; item < items; item += grid) {
                Region r;
                for (int region = 0; item_region(p, op, item, region, rt, r); ++region)
                    append_region(r, stage_chunks, units);
            }
        }
        offsets.push_back((unsigned)units.size());
    }
}

}  // namespace wsp
