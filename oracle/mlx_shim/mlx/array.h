// Shim forwarding header: see shim_core.h (test infrastructure only).
#pragma once
#include "shim_core.h"
