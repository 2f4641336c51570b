// gq_host.h — host-only helpers shared by the C++ (non-CUDA) parts of libgq.
#pragma once

#include <string>

#include "../../include/gq.h"

// Record a failure on the context (gq_last_error) and return the status.
int gq_set_error(gq_ctx *ctx, int status, const std::string &msg);
