// Launchers of the group-64 tcgen05 GEMM for W = 8 (all A, all tile widths).
#include "gemm_launch.cuh"

ACTUNE_INSTANTIATE_GEMM(8)
