// search_i8.cu -- search kernel instantiations for int8_t base vectors.
#include "plan.h"

namespace qv {
void bind_search_i8(Plan& pl) { bind_type<int8_t>(pl); }
}  // namespace qv
