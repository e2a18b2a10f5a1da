// TEST INFRASTRUCTURE ONLY -- minimal stand-in for ncnn's `net.h`: the
// reference's sampler and runtime-context headers include it for ncnn::Net and
// ncnn::Extractor, which the CPU sampler code never uses (declared only).
#pragma once

#include "mat.h"

namespace ncnn {
class Net;
class Extractor;
}  // namespace ncnn
