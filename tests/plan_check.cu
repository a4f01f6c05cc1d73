// plan_check: the table read's shared-memory plan for the Seoul tables at 1, 2, 4 and 8 inputs, made by the engine's
// own stage choice (mv_plan_stages in common.cuh, called with the MvArgs fields the engine sets: the Seoul shape's
// n_embd 2048 and d_conv 2, one CTA per SM of a 148-SM B200 at most). Host code only: prints one line per
// (table, inputs) with every region's offset, for the test to check that regions are aligned, ordered and inside one
// CTA's budget.
#include "../nunchi_b200/csrc/common.cuh"

#include <algorithm>
#include <cstdio>

using namespace imi;

int main() {
    struct T { const char *name; int rows, cols, pro, epi, hm; } ts[] = {
        { "in_proj", 6144, 2048, P_RESID_NORM, E_STORE, 0 }, { "out_proj", 2048, 2048, P_CONV, E_STORE, 0 },
        { "qkvg", 3104, 2048, P_RESID_NORM, E_STORE, 0 },     { "o", 2048, 2048, P_Q8IN, E_STORE, 0 },
        { "gate_up", 16384, 2048, P_RESID_NORM, E_SILU, 0 },   { "down", 2048, 8192, P_Q8IN, E_STORE, 0 },
        { "head", 97496, 2048, P_FINAL, E_HEAD, 0 },           { "q41_gate_up", 16384, 2048, P_RESID_NORM, E_SILU, 1 },
        { "q41_down", 2048, 8192, P_Q8IN, E_STORE, 1 },
    };
    for (auto &t : ts)
        for (int nc : { 1, 2, 4, 8 }) {
            const int gran = t.epi == E_SILU ? 2 : 1, unit = t.epi == E_SILU ? 64 : 1;
            const int rb = t.cols / 32 * (t.hm ? 20 : 18);
            const int units = t.rows / unit, grid = std::min(148, units), rows_cta = (units + grid - 1) / grid * unit;
            const int ab_len = t.epi == E_SILU ? (units + grid - 1) / grid * unit / 2 : 0;
            const int vb = mv_vb_len(t.pro, t.cols, 2048, nc, 2);
            const int full = std::max(gran, (std::min(64, MV_STAGE_BYTES / rb) / gran) * gran);
            MvArgs a = {};
            a.rows = t.rows; a.cols = t.cols; a.row_bytes = rb; a.unit = unit; a.ncol = nc; a.n_embd = 2048;
            a.ab_len = ab_len; a.d_conv = 2; a.has_m = t.hm;
            const int total = mv_plan_stages(a, t.pro, gran, grid);
            const int sr = total ? a.sr : 0, ns = total ? a.nstage : 0;
            const int budget = MV_SMEM_BUDGET;
            const MvPlan p = mv_plan(t.cols, sr ? sr : gran, nc, vb, ab_len, ns ? ns : 1, t.hm);
            printf("%s %d rb=%d full=%d rows_cta=%d sr=%d ns=%d stage=%d sstride=%d bar=%d xq=%d xd=%d xs=%d fs=%d dd=%d "
                   "vb=%d vo=%d ab=%d pc=%d red=%d total=%d budget=%d nc=%d nb=%d vb_len=%d ab_len=%d hm=%d\n",
                   t.name, nc, rb, full, rows_cta, sr, ns, p.stage, p.sstride, p.bar, p.xq, p.xd, p.xs, p.fs, p.dd,
                   p.vb, p.vo, p.ab, p.pc, p.red, p.total, budget, nc, t.cols / 32, vb, ab_len, t.hm);
        }
    return 0;
}
