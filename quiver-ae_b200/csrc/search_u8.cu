// search_u8.cu -- search kernel instantiations for uint8_t base vectors.
#include "plan.h"

namespace qv {
void bind_search_u8(Plan& pl) { bind_type<uint8_t>(pl); }
}  // namespace qv
