// search_f32.cu -- search kernel instantiations for float base vectors.
#include "plan.h"

namespace qv {
void bind_search_f32(Plan& pl) { bind_type<float>(pl); }
}  // namespace qv
