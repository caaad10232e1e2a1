// Prefill kernels (hsd/prefill.py): tile order, per-tile live unions and the grouped
// expert GEMM on the neuron-major layout.
#include "hsd_common.cuh"

HSD_DEFINE_STATUS(prefill)
