// pathpack_b200_internal.h — shared between the library's translation units.
#pragma once

#include "../../include/pathpack_b200.h"
