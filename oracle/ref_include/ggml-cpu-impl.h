// See ggml.h in this directory: the compute parameters the hook reads.
#pragma once
struct ggml_compute_params {
    int ith, nth;
};
