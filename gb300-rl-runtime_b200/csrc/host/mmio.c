/* mmio.c - the doorbell helpers are header inlines (mmio.h); this unit only
 * gives the library an object for them, like reference src/mmio.c. */
#include "mmio.h"

void
mmio_translation_unit_anchor(void)
{
}
