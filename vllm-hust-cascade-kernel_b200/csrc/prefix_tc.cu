// Stage-1 shared-prefix attention on tcgen05 (placeholder until the tile
// kernel lands: the planner routes > 16 rows here).
#include "kernels.h"

namespace cascade {
cudaError_t launch_paged_prefix_tc(const PagedAttnLaunch&, bool, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace cascade
