// Status codes shared by the device status word and the C-ABI return values.
#pragma once
#include "sae_b200.h"
