/* SwiftPM builds a C target from at least one source file; the module only
 * re-exports the C ABI of libtgsample.so (linked by name). */
#include "CTGSample.h"

int32_t ctgsample_abi_version(void) { return tg_abi_version(); }
