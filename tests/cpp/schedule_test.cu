// The decode kernel's weight-stream schedule (whispereacp_b200/csrc/schedule.h),
// checked on the host for op lists shaped like the decoder's: every unit
// starts 16-byte aligned, is a whole number of 16 bytes and fits a stage;
// the units of all CTAs together cover each weight matrix, the token table
// and each (window, head)'s cross keys and values exactly as often as the ops
// read them -- a product's weights once per row tile (or tensor-core row
// group), a fused cross query's head tiles once per (row, split), a window's
// keys once per row of that window -- with no byte skipped; and each op's L2
// prefetches are dealt out to exactly one CTA each.  No pointer is
// dereferenced: the weights are address ranges in a made-up arena.
//
//   schedule_test      prints "ok", or the first failure and exits 1
#include "../../whispereacp_b200/csrc/schedule.h"

#include <algorithm>
#include <cstdio>
#include <map>
#include <string>
#include <vector>

using namespace wsp;

namespace {

constexpr int kGrid = 148;

// Address ranges standing in for device allocations.
struct Arena {
    size_t next = (size_t)1 << 40;
    const unsigned char* take(size_t bytes) {
        const size_t at = next;
        next += (bytes + 4095) / 4096 * 4096 + 4096;
        return reinterpret_cast<const unsigned char*>(at);
    }
};

struct Range {
    std::string what;
    size_t base, size;
    int times;
};

std::string failure;
bool fail(const std::string& s) {
    if (failure.empty()) failure = s;
    return false;
}

bool check(const std::string& name, const StepParams& p, const std::vector<StepOp>& ops, int rt,
           const std::vector<Range>& ranges) {
    std::vector<ScheduleEntry> units;
    std::vector<unsigned> offsets;
    build_schedule(p, ops, kGrid, rt, units, offsets);
    if (offsets.size() != (size_t)kGrid + 1 || offsets.back() != units.size())
        return fail(name + ": the offsets do not delimit every CTA's schedule");
    // Every unit's shape.
    for (size_t i = 0; i < units.size(); ++i) {
        const ScheduleEntry& e = units[i];
        if (e.bytes & kPrefetchOnly) continue;
        if (e.source % 16 != 0 || e.bytes % 16 != 0 || e.bytes == 0 || e.bytes > (unsigned long long)p.stage_bytes)
            return fail(name + ": unit " + std::to_string(i) + " is misaligned, empty or larger than a stage");
    }
    // Coverage: each range read exactly `times` times, byte for byte, and no
    // unit outside every range.
    size_t in_ranges = 0, unit_bytes = 0;
    for (const ScheduleEntry& e : units)
        if (!(e.bytes & kPrefetchOnly)) unit_bytes += (size_t)e.bytes;
    for (const Range& r : ranges) {
        std::vector<std::pair<size_t, int>> events;
        for (const ScheduleEntry& e : units) {
            if (e.bytes & kPrefetchOnly) continue;
            const size_t lo = (size_t)e.source, hi = lo + (size_t)e.bytes;
            if (hi <= r.base || lo >= r.base + r.size) continue;
            if (lo < r.base || hi > r.base + r.size) return fail(name + ": a unit straddles the edge of " + r.what);
            events.push_back({lo, +1});
            events.push_back({hi, -1});
            in_ranges += hi - lo;
        }
        std::sort(events.begin(), events.end());
        size_t at = r.base;
        int count = 0;
        for (size_t i = 0; i < events.size();) {
            const size_t x = events[i].first;
            if (x > at && count != r.times)
                return fail(name + ": " + r.what + " bytes " + std::to_string(at - r.base) + ".." +
                            std::to_string(x - r.base) + " are read " + std::to_string(count) + " times, not " +
                            std::to_string(r.times));
            for (; i < events.size() && events[i].first == x; ++i) count += events[i].second;
            at = x;
        }
        if (at != r.base + r.size || (events.empty() && r.times != 0))
            return fail(name + ": the end of " + r.what + " is never read");
    }
    if (in_ranges != unit_bytes) return fail(name + ": units read bytes outside every weight range");
    // Prefetches: the multiset over all CTAs equals the ops' own lists.
    std::map<std::pair<unsigned long long, unsigned long long>, int> wanted, dealt;
    for (const StepOp& op : ops) {
        std::vector<std::pair<const void*, unsigned long long>> pf;
        op_prefetches(p, op, pf);
        for (const auto& e : pf) ++wanted[{(unsigned long long)(size_t)e.first, e.second}];
    }
    for (const ScheduleEntry& e : units)
        if (e.bytes & kPrefetchOnly) ++dealt[{e.source, e.bytes & ~kPrefetchOnly}];
    if (wanted != dealt) return fail(name + ": the L2 prefetches are not dealt out once each");
    return true;
}

int round16(int n) { return (n + 15) / 16 * 16; }

StepOp product(const unsigned char* weight, int n, int kp, const float* bias) {
    StepOp o{};
    o.kind = kOpProduct;
    o.weight = weight;
    o.n = n;
    o.kp = kp;
    o.bias = bias;
    return o;
}

// Fragment-packed matrix bytes: 16-row tiles of kp / 32 one-KB chunks.
size_t packed_bytes(int n, int kp) { return (size_t)((n + 15) / 16) * (kp / 32) * 1024; }
// Tensor-core matrix bytes: 128-row tiles of kp / 64 16-KB blocks.
size_t umma_bytes(int n, int kp) { return (size_t)((n + 127) / 128) * (kp / 64) * 16384; }

struct Shape {
    int width, heads, ffn, vocabulary, keys;
};

// The few-row mma.sync form: the attention ops apply the out-projections,
// the cross attention computes its own query, fc2 splits its K into parts.
bool few_rows(const std::string& name, const Shape& s, int windows, int tokens, int layers) {
    Arena a;
    const int d = s.width, H = s.heads, D = d / H, kpd = d, kpf = s.ffn;
    StepParams p{};
    p.windows = windows;
    p.tokens = tokens;
    p.rows = windows * tokens;
    p.width = d;
    p.heads = H;
    p.head_width = D;
    p.vocabulary = s.vocabulary;
    p.kpd = kpd;
    p.out_rows = windows;
    p.stage_bytes = std::max(16384, 16 * kpd * 2);
    p.token_table = a.take(packed_bytes(s.vocabulary, kpd));
    p.final_gamma = reinterpret_cast<const float*>(a.take(4 * d));
    p.final_beta = reinterpret_cast<const float*>(a.take(4 * d));
    p.mask = reinterpret_cast<const float*>(a.take(4 * (size_t)s.vocabulary));
    const int chunk = p.stage_bytes / (4 * D), units = (s.keys + chunk - 1) / chunk, splits = 4;
    const long long head_block = (long long)s.keys * 2 * D;
    const unsigned char* keys = a.take((size_t)layers * windows * H * head_block * 2);
    std::vector<Range> ranges{{"the token table", (size_t)p.token_table, packed_bytes(s.vocabulary, kpd), 1}};
    std::vector<StepOp> ops;
    StepOp e{};
    e.kind = kOpEmbed;
    ops.push_back(e);
    for (int l = 0; l < layers; ++l) {
        const std::string at = " of layer " + std::to_string(l);
        auto bias = [&](int n) { return reinterpret_cast<const float*>(a.take(4 * (size_t)n)); };
        StepOp qkv = product(a.take(packed_bytes(H * round16(3 * D), kpd)), H * round16(3 * D), kpd, bias(3 * d));
        qkv.gamma = bias(d);
        qkv.beta = bias(d);
        ranges.push_back({"q/k/v" + at, (size_t)qkv.weight, packed_bytes(qkv.n, kpd), 1});
        ops.push_back(qkv);
        StepOp self{};
        self.kind = kOpSelfAttention;
        self.out_weight = a.take(packed_bytes(d, kpd));
        ops.push_back(self);
        StepOp cross = product(a.take(packed_bytes(H * round16(D), kpd)), H * round16(D), kpd, bias(d));
        cross.kind = kOpCrossAttention;
        cross.gamma = bias(d);
        cross.beta = bias(d);
        cross.addend_bias = bias(d);
        cross.keys = keys + (size_t)l * windows * H * head_block * 2;
        cross.key_stride = 2 * D;
        cross.head_stride = head_block;
        cross.window_stride = (long long)H * head_block;
        cross.key_count = s.keys;
        cross.chunk = chunk;
        cross.splits = splits;
        cross.span = (units + splits - 1) / splits;
        cross.value_bias = bias(d);
        cross.out_weight = a.take(packed_bytes(d, kpd));
        // A fused query: each (row, head, split) item reads its head's q tiles.
        for (int h = 0; h < H; ++h)
            ranges.push_back({"head " + std::to_string(h) + "'s cross query" + at,
                              (size_t)cross.weight + (size_t)h * (round16(D) / 16) * (kpd / 32) * 1024,
                              (size_t)(round16(D) / 16) * (kpd / 32) * 1024, p.rows * splits});
        for (int b = 0; b < windows; ++b)
            for (int h = 0; h < H; ++h)
                ranges.push_back({"window " + std::to_string(b) + " head " + std::to_string(h) + "'s cross keys" + at,
                                  (size_t)cross.keys + ((size_t)b * cross.window_stride + (size_t)h * head_block) * 2,
                                  (size_t)head_block * 2, tokens});
        ops.push_back(cross);
        StepOp up = product(a.take(packed_bytes(s.ffn, kpd)), s.ffn, kpd, bias(s.ffn));
        up.gamma = bias(d);
        up.beta = bias(d);
        ranges.push_back({"fc1" + at, (size_t)up.weight, packed_bytes(s.ffn, kpd), 1});
        ops.push_back(up);
        StepOp down = product(a.take(packed_bytes(d, kpf)), d, kpf, bias(d));
        down.kparts = 4;
        ranges.push_back({"fc2" + at, (size_t)down.weight, packed_bytes(d, kpf), 1});
        ops.push_back(down);
    }
    StepOp logits{};
    logits.kind = kOpLogits;
    ops.push_back(logits);
    return check(name, p, ops, 8, ranges);
}

// The batched mma.sync form: norm ops, plain products read by every row
// tile, the cross attention over the CTA's items.
bool batched_mma(const std::string& name, const Shape& s, int windows, int rt) {
    Arena a;
    const int d = s.width, H = s.heads, D = d / H, kpd = d, kpf = s.ffn;
    StepParams p{};
    p.windows = windows;
    p.tokens = 1;
    p.rows = windows;
    p.width = d;
    p.heads = H;
    p.head_width = D;
    p.vocabulary = s.vocabulary;
    p.kpd = kpd;
    p.out_rows = windows;
    p.stage_bytes = std::max(16384, 16 * kpd * 2);
    p.token_table = a.take(packed_bytes(s.vocabulary, kpd));
    const int row_tiles = (windows + rt - 1) / rt;
    std::vector<Range> ranges{{"the token table", (size_t)p.token_table, packed_bytes(s.vocabulary, kpd), row_tiles}};
    std::vector<StepOp> ops;
    auto bias = [&](int n) { return reinterpret_cast<const float*>(a.take(4 * (size_t)n)); };
    auto add_product = [&](const char* what, int n, int kp) {
        StepOp o = product(a.take(packed_bytes(n, kp)), n, kp, bias(n));
        ranges.push_back({what, (size_t)o.weight, packed_bytes(n, kp), row_tiles});
        ops.push_back(o);
    };
    StepOp norm{};
    norm.kind = kOpNorm;
    norm.gamma = bias(d);
    norm.beta = bias(d);
    ops.push_back(norm);
    add_product("q/k/v", H * round16(3 * D), kpd);
    add_product("out-projection", d, kpd);
    add_product("cross query", H * round16(D), kpd);
    const int chunk = p.stage_bytes / (4 * D), units = (s.keys + chunk - 1) / chunk;
    const long long head_block = (long long)s.keys * 2 * D;
    StepOp cross{};
    cross.kind = kOpCrossAttention;
    cross.keys = a.take((size_t)windows * H * head_block * 2);
    cross.key_stride = 2 * D;
    cross.head_stride = head_block;
    cross.window_stride = (long long)H * head_block;
    cross.key_count = s.keys;
    cross.chunk = chunk;
    cross.splits = 1;
    cross.span = units;
    cross.value_bias = bias(d);
    ranges.push_back({"the cross keys", (size_t)cross.keys, (size_t)windows * H * head_block * 2, 1});
    ops.push_back(cross);
    add_product("fc1", s.ffn, kpd);
    add_product("fc2 (tiles larger than a stage)", d, kpf);
    StepOp logits{};
    logits.kind = kOpLogits;
    ops.push_back(logits);
    return check(name, p, ops, rt, ranges);
}

// The tensor-core form: products split over K, tcgen05 logits.
bool tensor_core(const std::string& name, const Shape& s, int windows, int umma_rows, int stage_bytes) {
    Arena a;
    const int d = s.width, H = s.heads, D = d / H;
    StepParams p{};
    p.windows = windows;
    p.tokens = 1;
    p.rows = windows;
    p.width = d;
    p.heads = H;
    p.head_width = D;
    p.vocabulary = s.vocabulary;
    p.kpd = d;
    p.out_rows = windows;
    p.umma = 1;
    p.umma_rows = umma_rows;
    p.stage_bytes = stage_bytes;
    p.umma_blocks = std::max(1, stage_bytes / 16384);
    p.token_table = a.take(umma_bytes(s.vocabulary, d));
    const int groups = (windows + umma_rows - 1) / umma_rows;
    std::vector<Range> ranges{
        {"the token table", (size_t)p.token_table, umma_bytes(s.vocabulary, d), (windows + 127) / 128}};
    std::vector<StepOp> ops;
    auto bias = [&](int n) { return reinterpret_cast<const float*>(a.take(4 * (size_t)n)); };
    auto add_product = [&](const char* what, int n, int kp, int ksplit) {
        StepOp o = product(a.take(umma_bytes(n, kp)), n, kp, bias(n));
        // As the host sizes splits: whole blocks each, none empty.
        const int kblocks = kp / 64, per = (kblocks + ksplit - 1) / ksplit;
        o.ksplit = (kblocks + per - 1) / per;
        ranges.push_back({what, (size_t)o.weight, umma_bytes(n, kp), groups});
        ops.push_back(o);
    };
    add_product("q/k/v (6 splits of 16 blocks)", 3 * d, d, 6);
    add_product("out-projection", d, d, 16);
    add_product("fc1", s.ffn, d, 4);
    add_product("fc2", d, s.ffn, 16);
    add_product("a product in one piece", d, d, 1);
    const int chunk = stage_bytes / (4 * D), units = (s.keys + chunk - 1) / chunk;
    const long long head_block = (long long)s.keys * 2 * D;
    StepOp cross{};
    cross.kind = kOpCrossAttention;
    cross.keys = a.take((size_t)windows * H * head_block * 2);
    cross.key_stride = 2 * D;
    cross.head_stride = head_block;
    cross.window_stride = (long long)H * head_block;
    cross.key_count = s.keys;
    cross.chunk = chunk;
    cross.splits = 1;
    cross.span = units;
    ranges.push_back({"the cross keys", (size_t)cross.keys, (size_t)windows * H * head_block * 2, 1});
    ops.push_back(cross);
    StepOp logits{};
    logits.kind = kOpLogits;
    ops.push_back(logits);
    return check(name, p, ops, 8, ranges);
}

}  // namespace

int main() {
    const Shape tiny{384, 6, 1536, 51864, 1500}, base{512, 8, 2048, 51864, 1500}, small{768, 12, 3072, 51864, 1500},
        medium{1024, 16, 4096, 51864, 1500}, large{1280, 20, 5120, 51866, 1500};
    const bool ok = few_rows("tiny.en, 1 window", tiny, 1, 1, 2) && few_rows("base.en, 1 window", base, 1, 1, 2) &&
                    few_rows("base.en, the 2-token prompt", base, 1, 2, 1) &&
                    few_rows("base.en, 4 windows", base, 4, 1, 1) &&
                    batched_mma("small.en, 24 windows, 16-row tiles", small, 24, 16) &&
                    batched_mma("base.en, 16 windows, 32-row tiles", base, 16, 32) &&
                    tensor_core("medium.en, 64 windows", medium, 64, 64, 32768) &&
                    tensor_core("large-v3, 128 windows", large, 128, 128, 40960) &&
                    tensor_core("small.en, 200 windows (two row groups)", small, 200, 128, 24576);
    if (!ok) {
        std::printf("FAIL %s\n", failure.c_str());
        return 1;
    }
    std::printf("ok\n");
    return 0;
}
