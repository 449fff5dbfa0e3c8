// Routed attention (placeholder until the tcgen05 kernel lands).
#include "sm100.cuh"
RC_DEVICE_ERROR_ACCESSOR(attention)
