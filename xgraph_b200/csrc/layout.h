// Internal: the public ABI types (XgState, XgLayout, XgOptions) shared by the kernels,
// the C ABI and the host-seam build.
#pragma once
#include "../../include/xgraph_b200.h"
