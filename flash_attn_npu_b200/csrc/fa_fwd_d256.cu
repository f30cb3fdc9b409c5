// Kernel instantiations for head_dim = 256 (see fa_fwd_dispatch.cuh for the tile table).
#define FA_HEAD_DIM 256
#include "fa_fwd_dispatch.cuh"
