// SET regrow draws on the host, bit-identical to the reference's per-row
//     rng.choice(pool, size=n_grow, replace=False)
// loop (sparselab/router.py:457-470) on a numpy Generator(PCG64), without a
// Python call per row.
//
// The draws follow numpy's published Generator algorithms (numpy 2.3,
// numpy/random/_generator.pyx `choice`, numpy/random/src/distributions
// `random_bounded_uint64`, numpy/random/src/pcg64):
//   * PCG64: 128-bit LCG (multiplier 0x2360ed051fc65da4_4385df649fccf645),
//     state advanced before each output, XSL-RR output
//     rotr64(hi ^ lo, hi >> 58); 32-bit draws take the low half of a 64-bit
//     output and keep the high half for the next 32-bit draw (has_uint32 /
//     uinteger in the generator state).
//   * bounded integers in [0, rng] (rng < 2^32 - 1): Lemire's
//     multiply-shift with rejection on a 32-bit draw; rng = 2^32 - 1: a raw
//     32-bit draw; rng = 0: no draw.  Wider ranges use the 64-bit variant.
//   * choice without replacement, shuffle=True: for pool > 10000 and
//     size > pool / 50 a partial Fisher-Yates ("tail shuffle") of
//     0..pool-1 whose last `size` entries are the result; otherwise Robert
//     Floyd's sampling (j from pool-size to pool-1: draw v in [0, j], take v
//     unless already taken, else take j) followed by a Fisher-Yates shuffle
//     of the result (i from size-1 down to 1, swap with a draw in [0, i]).
// The generator state is read from and written back to the caller's numpy
// Generator, so later draws (and checkpoints of the state) continue exactly.
#include <cstdint>
#include <string>
#include <algorithm>
#include <vector>

#include "common.cuh"

namespace slb {
namespace {

using u128 = unsigned __int128;

struct Pcg64 {
    u128 state, inc;
    bool has32;
    uint32_t uint32;

    uint64_t next64() {
        const u128 mult = (static_cast<u128>(0x2360ed051fc65da4ULL) << 64) | 0x4385df649fccf645ULL;
        state = state * mult + inc;
        const uint64_t hi = static_cast<uint64_t>(state >> 64), lo = static_cast<uint64_t>(state);
        const unsigned rot = static_cast<unsigned>(hi >> 58);
        const uint64_t x = hi ^ lo;
        return (x >> rot) | (x << ((64u - rot) & 63u));
    }
    uint32_t next32() {
        if (has32) {
            has32 = false;
            return uint32;
        }
        const uint64_t n = next64();
        has32 = true;
        uint32 = static_cast<uint32_t>(n >> 32);
        return static_cast<uint32_t>(n & 0xffffffffu);
    }
    // Uniform integer in [0, rng].
    uint64_t bounded(uint64_t rng) {
        if (rng == 0) return 0;
        if (rng <= 0xffffffffULL) {
            if (rng == 0xffffffffULL) return next32();
            const uint32_t excl = static_cast<uint32_t>(rng) + 1u;
            uint64_t m = static_cast<uint64_t>(next32()) * excl;
            uint32_t left = static_cast<uint32_t>(m);
            if (left < excl) {
                const uint32_t thr = (0xffffffffu - static_cast<uint32_t>(rng)) % excl;
                while (left < thr) {
                    m = static_cast<uint64_t>(next32()) * excl;
                    left = static_cast<uint32_t>(m);
                }
            }
            return m >> 32;
        }
        if (rng == 0xffffffffffffffffULL) return next64();
        const uint64_t excl = rng + 1;
        u128 m = static_cast<u128>(next64()) * excl;
        uint64_t left = static_cast<uint64_t>(m);
        if (left < excl) {
            const uint64_t thr = (0xffffffffffffffffULL - rng) % excl;
            while (left < thr) {
                m = static_cast<u128>(next64()) * excl;
                left = static_cast<uint64_t>(m);
            }
        }
        return static_cast<uint64_t>(m >> 64);
    }
};

// rng.choice(pop, size=size, replace=False) -> out[0 .. size).
// `mark` (at least pop entries) and `epoch` implement Floyd's "taken" set:
// v is taken in this call iff mark[v] == epoch.
void choice_no_replace(Pcg64& g, int64_t pop, int64_t size, int32_t* out,
                       std::vector<int64_t>& work, std::vector<uint32_t>& mark, uint32_t& epoch) {
    if (pop > 10000 && size > pop / 50) {
        work.resize(static_cast<size_t>(pop));
        for (int64_t i = 0; i < pop; ++i) work[i] = i;
        const int64_t first = pop - size > 1 ? pop - size : 1;
        for (int64_t i = pop - 1; i >= first; --i) {
            const int64_t j = static_cast<int64_t>(g.bounded(static_cast<uint64_t>(i)));
            const int64_t t = work[j];
            work[j] = work[i];
            work[i] = t;
        }
        for (int64_t k = 0; k < size; ++k) out[k] = static_cast<int32_t>(work[pop - size + k]);
        return;
    }
    work.resize(static_cast<size_t>(size));
    if (static_cast<int64_t>(mark.size()) < pop) mark.assign(static_cast<size_t>(pop), 0u);
    if (++epoch == 0) {  // wrapped: clear
        std::fill(mark.begin(), mark.end(), 0u);
        epoch = 1;
    }
    for (int64_t j = pop - size; j < pop; ++j) {
        const int64_t v = static_cast<int64_t>(g.bounded(static_cast<uint64_t>(j)));
        const int64_t take = mark[v] != epoch ? v : j;
        mark[take] = epoch;
        work[j - pop + size] = take;
    }
    for (int64_t i = size - 1; i >= 1; --i) {
        const int64_t j = static_cast<int64_t>(g.bounded(static_cast<uint64_t>(i)));
        const int64_t t = work[j];
        work[j] = work[i];
        work[i] = t;
    }
    for (int64_t k = 0; k < size; ++k) out[k] = static_cast<int32_t>(work[k]);
}

}  // namespace
}  // namespace slb

using namespace slb;

extern "C" int sl_set_regrow_draws(uint64_t* pcg_state, int32_t* has_uint32, uint32_t* uinteger,
                                   int64_t nrows, const int32_t* n_live, const int32_t* n_keep,
                                   int64_t ncols, int32_t* counts, int32_t* ranks,
                                   int64_t ranks_cap, int64_t* n_ranks) {
    SL_REQUIRE(pcg_state != nullptr && has_uint32 != nullptr && uinteger != nullptr,
               "sl_set_regrow_draws", "NULL generator state");
    SL_REQUIRE(nrows >= 0 && ncols >= 0, "sl_set_regrow_draws", "negative size");
    SL_REQUIRE(nrows == 0 || (n_live != nullptr && n_keep != nullptr && counts != nullptr),
               "sl_set_regrow_draws", "NULL row array");
    SL_REQUIRE(n_ranks != nullptr && (ranks_cap == 0 || ranks != nullptr), "sl_set_regrow_draws",
               "NULL output");
    Pcg64 g;
    g.state = (static_cast<u128>(pcg_state[0]) << 64) | pcg_state[1];
    g.inc = (static_cast<u128>(pcg_state[2]) << 64) | pcg_state[3];
    g.has32 = *has_uint32 != 0;
    g.uint32 = *uinteger;
    std::vector<int64_t> work;
    std::vector<uint32_t> mark;
    uint32_t epoch = 0;
    int64_t used = 0;
    for (int64_t i = 0; i < nrows; ++i) {
        counts[i] = 0;
        const int64_t live = n_live[i], keep = n_keep[i];
        if (live <= 0) continue;
        SL_REQUIRE(keep >= 0 && keep <= live && keep <= ncols, "sl_set_regrow_draws",
                   "row " + std::to_string(i) + ": survivors out of range");
        const int64_t pool = ncols - keep, drop = live - keep;
        if (pool == 0 || drop == 0) continue;
        const int64_t grow = drop < pool ? drop : pool;
        SL_REQUIRE(used + grow <= ranks_cap, "sl_set_regrow_draws", "ranks buffer too small");
        choice_no_replace(g, pool, grow, ranks + used, work, mark, epoch);
        counts[i] = static_cast<int32_t>(grow);
        used += grow;
    }
    pcg_state[0] = static_cast<uint64_t>(g.state >> 64);
    pcg_state[1] = static_cast<uint64_t>(g.state);
    *has_uint32 = g.has32 ? 1 : 0;
    *uinteger = g.uint32;
    *n_ranks = used;
    return SL_OK;
}
