// Verify attention, tensor-memory path (tcgen05 MMA + TMEM accumulators).
// Placeholder until the sm_100a tensor-core kernel lands: reports itself as
// unavailable so the planner always takes the warp-MMA path.
#include "attn_kernels.cuh"
#include "common.cuh"

namespace tv {

bool tc_supported(int, int, int, bool, int) { return false; }
int tc_tile_keys() { return 128; }
int tc_rows_per_cta() { return 256; }
int launch_attn_tc(const AttnParams&, int, int, cudaStream_t) { return TV_ERR_UNSUPPORTED; }

}  // namespace tv
