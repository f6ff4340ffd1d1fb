// knn_tc.cu -- tcgen05 (5th-generation tensor core) distance-tile engine.
#include "knn_common.cuh"

namespace fdb {

bool tc_engine_supported(int) { return false; }

void launch_tile_round_tc(const TileRound&, int, int, cudaStream_t)
{
    throw Error(FDB200_EINVAL, "the tcgen05 engine is not available in this build");
}

}  // namespace fdb
