// Device-side helpers plus the launcher declarations.
#pragma once

#include "common.cuh"
#include "launch.h"
