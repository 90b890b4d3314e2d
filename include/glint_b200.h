/* Library identity and the attach-ABI version string.
 *
 * p7_abi_version() answers "p7_attach_abi_v1" exactly as the reference's
 * cuda/p7_abi.c:3-11 does (attach/ABI_VERSION); the glint entry points are
 * additive to that ABI, which lists no glint symbols (attach/CONTRACT.md:10-16).
 */
#ifndef GLINT_B200_H_
#define GLINT_B200_H_
#ifdef __cplusplus
extern "C" {
#endif
const char *p7_abi_version(void);
/* "glint_b200 <version> sm_100a" */
const char *glint_b200_version(void);
/* Error word of the current device, ORed by kernels that stopped instead of
 * hanging or faulting: 1 = a bounded wait on a pipeline barrier or a peer's signal
 * ran out; 2 = a kernel found its shared-memory ring misaligned for a tensor copy
 * and issued none.  0 when none.  Synchronous.  clear != 0 resets it. */
int glint_kernel_error(int clear);
#ifdef __cplusplus
}
#endif
#endif
