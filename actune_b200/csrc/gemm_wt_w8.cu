// Launchers of the weights-in-TMEM group-64 GEMM for W = 8 (all A, all token tiles).
#define ACTUNE_WT_LAUNCH_DEFINITIONS
#include "gemm_wt.cuh"

ACTUNE_INSTANTIATE_WT(8)
