// Kernel instantiations for head_dim = 128 (see fa_fwd_dispatch.cuh for the tile table).
#define FA_HEAD_DIM 128
#include "fa_fwd_dispatch.cuh"
