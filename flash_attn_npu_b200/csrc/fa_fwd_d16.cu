// Kernel instantiations for head_dim = 16 (see fa_fwd_dispatch.cuh for the tile table).
#define FA_HEAD_DIM 16
#include "fa_fwd_dispatch.cuh"
