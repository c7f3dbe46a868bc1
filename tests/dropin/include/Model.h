// The reference's Model.h mapped onto this library's header (drop-in shim for its tests).
#pragma once
#include "ModelConfig.h"
#include "veda/train.hpp"
