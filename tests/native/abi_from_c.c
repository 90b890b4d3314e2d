/* The C ABI used from plain C (C11): every public header compiles in a C
 * translation unit, the library links, and the device-free helpers answer as
 * the reference's do (include/glint_encode.h:17-18, cuda/p7_abi.c:3-11). */
#include <stdio.h>
#include <string.h>

#include "../../include/glint_b200.h"
#include "../../include/glint_cells.h"
#include "../../include/glint_encode.h"
#include "../../include/glint_htile.h"
#include "../../include/glint_meta.h"
#include "../../include/glint_plug_streamer.h"

int main(void)
{
    int bad = 0;
    bad += glint_encode_n_packed(7) != 4;
    bad += glint_encode_n_absmax(65, 64) != 2;
    bad += glint_encode_n_absmax(5, 0) != 0;
    bad += strcmp(p7_abi_version(), "p7_attach_abi_v1") != 0;
    bad += glint_plug_streamer_start(NULL) != -1;
    bad += glint_plug_streamer_host_buffer(NULL, 0) != NULL;
    bad += GLINT_CELLS[0][0] >= GLINT_CELLS[0][1];
    bad += sizeof(GlintStreamerStats) != 8 + 8 + 64 * 8 + 8;
    printf("%s\n", bad ? "FAIL" : "OK");
    return bad != 0;
}
