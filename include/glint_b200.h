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
/* Error word of the current device, set by a kernel whose bounded wait on a
 * pipeline barrier ran out (1 = timeout); 0 when none.  Synchronous.  clear != 0
 * resets it. */
int glint_kernel_error(int clear);
#ifdef __cplusplus
}
#endif
#endif
