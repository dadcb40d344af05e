// gemm_plan.h — shared-memory plan of k_gemm_tc (host arithmetic only, no CUDA types), kept in
// its own header so that the CPU tests compile and check it.
//
// Ring depths within ~222 KB: 4 stages (activation tile + decoded weights) if at least 4 raw
// chunks still fit, else 3; the raw ring takes the rest (up to 12 chunks). The two decoder
// groups take alternate k steps and wait on a raw slot by phase parity, which is exact only
// while the slot's barrier is at most one phase behind, i.e. while the slot's previous chunk has
// landed. With an even ring that chunk is the waiting group's own, which it consumed before.
// With an odd ring it is the other group's; a group waiting for chunk k has finished chunk k - 2,
// whose stage wait means the MMA consumed chunk k - 2 - NS, so every chunk up to there has
// landed: an odd ring is exact only from NS + 2 slots on. Below that the parity test can pass on
// the wrong phase (a torn chunk decoded, the ring's arrival counts off by a group), so such a
// ring gives up one slot.
#pragma once

#include <cstddef>

namespace jv {

struct GemmRingPlan {
    int ns = 0;          // stages: decoded-weight tile (16 KB) + activation tile (bn x 128 B)
    int nr = 0;          // raw-chunk slots
    int b_off = 0;       // byte offsets inside the 1024-aligned dynamic shared memory (A at 0)
    int raw_off = 0;
    int bar_off = 0;
    size_t smem = 0;     // dynamic shared memory to request
};

constexpr size_t GEMM_SMEM_BUDGET = 222 * 1024;

// The plan for token tile bn and raw chunk size cb; false when fewer than two raw slots fit.
inline bool gemm_ring_plan(int bn, int cb, GemmRingPlan* p) {
    const size_t stage = 16384 + (size_t)bn * 128;
    p->ns = (stage * 4 + 4 * (size_t)cb <= GEMM_SMEM_BUDGET) ? 4 : 3;
    if (stage * p->ns > GEMM_SMEM_BUDGET) return false;
    const size_t fit = (GEMM_SMEM_BUDGET - stage * p->ns) / (size_t)cb;
    p->nr = (int)(fit < 12 ? fit : 12);
    if (p->nr % 2 == 1 && p->nr < p->ns + 2) p->nr -= 1;
    if (p->nr < 2) return false;
    p->b_off = 16384 * p->ns;
    p->raw_off = p->b_off + bn * 128 * p->ns;
    p->bar_off = (p->raw_off + cb * p->nr + 15) & ~15;
    // barriers: raw full/empty, stage b_full/a_full/empty, two accumulators' full/empty and the
    // drain barrier; then the TMEM slot and a flag, and the 1024-byte alignment slack
    p->smem = (size_t)p->bar_off + 8 * (2 * p->nr + 3 * p->ns + 5) + 16 + 1024;
    return true;
}

}  // namespace jv
