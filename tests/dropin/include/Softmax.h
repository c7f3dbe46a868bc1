// The reference's Softmax.h mapped onto this library's header (drop-in shim for its tests).
#pragma once
#include "veda/ops.hpp"
