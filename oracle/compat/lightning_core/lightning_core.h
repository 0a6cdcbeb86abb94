/* Include-path stand-in used only to compile the reference's own C example
 * (examples/lightning_core_c_api.c, unchanged, from the reference tree) against this build's C
 * ABI: the example includes "lightning_core/lightning_core.h", whose runtime part is repeated
 * symbol for symbol in include/lc_b200.h. */
#include "../../../include/lc_b200.h"
