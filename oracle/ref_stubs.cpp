// Two symbols the reference's order.cpp links against whose own translation units
// (carbon/src/score.cpp, carbon/src/engine.cpp) pull in the whole engine.  Line
// recognition never calls either; they throw if anything does.
// TEST INFRASTRUCTURE ONLY (oracle/_ref).
#include <span>
#include <string>
#include <string_view>
#include <vector>

#include "carbon/engine.h"
#include "carbon/error.h"
#include "carbon/score.h"

namespace carbon {

std::u32string code_points(std::string_view) { throw Error("oracle/_ref: code_points is not built"); }

std::vector<size_t> reading_order(std::span<const LineBox>) { throw Error("oracle/_ref: reading_order is not built"); }

}  // namespace carbon
