// Kernel instantiations for head_dim = 64 (see fa_fwd_dispatch.cuh for the tile table).
#define FA_HEAD_DIM 64
#include "fa_fwd_dispatch.cuh"
