/*
 * Stand-in for ggml's internal header as the reference's src/xdna-exec.cpp
 * uses it: the graph's node list (it reads n_nodes and nodes directly).
 * TEST INFRASTRUCTURE ONLY.
 */
#pragma once

#include "ggml.h"

struct ggml_cgraph {
    int size;
    int n_nodes;
    int n_leafs;
    struct ggml_tensor **nodes;
    struct ggml_tensor **leafs;
};
