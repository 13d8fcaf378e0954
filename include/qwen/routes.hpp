// qwen/routes.hpp -- drop-in for the reference's src/routes.hpp.
//
// A caller built against the reference (namespace qwen, #include "routes.hpp")
// puts include/qwen/ ahead of the reference's src/ on its include path and
// links libqwen_moe_b200.so instead of compiling src/routes.cpp: the names,
// signatures, exceptions and allocation rules are the reference's
// (src/routes.hpp:9-65), implemented by qmoe::RouteGroups.
#pragma once

#include "../qmoe/routes.hpp"

namespace qwen {
using qmoe::RouteAssignment;
using qmoe::RouteGroups;
}  // namespace qwen
