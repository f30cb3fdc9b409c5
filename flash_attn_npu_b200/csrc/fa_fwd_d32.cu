// Kernel instantiations for head_dim = 32 (see fa_fwd_dispatch.cuh for the tile table).
#define FA_HEAD_DIM 32
#include "fa_fwd_dispatch.cuh"
