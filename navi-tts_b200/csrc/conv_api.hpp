// Host-only declaration of the one-shot convolution entry (navi_conv1d): packs the weight,
// runs conv::launch once on the device's stream and waits for it.
#pragma once

#include "../../include/navi_b200.h"
#include "runtime.hpp"

namespace navi {

int conv_once(const Device & dev, const navi_conv_args & a);

} // namespace navi
