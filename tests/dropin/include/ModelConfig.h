// The reference's ModelConfig.h mapped onto this library's header (drop-in shim for its tests):
// io::ModelConfig is the same struct as train::ModelConfig here (the reference's field names).
#pragma once
#include "veda/train.hpp"
namespace veda::io
{
using ModelConfig = veda::train::ModelConfig;
}
