// Routed-expert MLP (src/moe.zig:998-1228).
#include "model.cuh"

namespace ditch {

int moe_mlp(ditch_cuda_model *m, Layer &L, int li, int n) {
    (void)m;
    (void)L;
    (void)li;
    (void)n;
    set_error("MoE layers are not available in this build");
    return DITCH_CUDA_UNSUPPORTED;
}

}  // namespace ditch
