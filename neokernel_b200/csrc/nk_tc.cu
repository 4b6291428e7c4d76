// tcgen05/TMEM tensor-core family (swap-AB: weight rows are the MMA's M = 128 operand,
// decode tokens are its N). Not selectable yet: nk_plan_make refuses NK_KIND_TC.
#include "nk_common.cuh"

namespace nk {

int launch_tc(const nk_plan& p, const GemmArgs& a, cudaStream_t s) {
    (void)p; (void)a; (void)s;
    return NK_ERR_PLAN;
}

}  // namespace nk
