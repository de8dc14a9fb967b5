// Baked results of the offline tile sweep (one entry per measured dispatch
// shape). Regenerated from the sweep's JSON output; shapes that are not
// listed fall back to the planner's cost model.
#include "planner.h"

namespace hxb {

const TunedGemm kTunedGemms[] = {
#include "tile_table.inc"
    {0, 0, 0, -1, 0, 0, 0, 0},  // sentinel, never matches (bmode -1)
};
const int kNumTunedGemms = sizeof(kTunedGemms) / sizeof(kTunedGemms[0]) - 1;

}  // namespace hxb
