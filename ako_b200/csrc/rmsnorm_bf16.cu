// Instantiates the RMSNorm launchers for one storage dtype.
#define AKO_RMS_INSTANTIATING
#include "rmsnorm.cuh"

namespace ako_b200 {
AKO_RMS_DECLARE(__nv_bfloat16, )
}  // namespace ako_b200
