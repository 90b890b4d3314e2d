/* GLINT codebook: GLINT_CELLS[hole][plug] and the 16-entry parent table.
 *
 * Values are the reference codebook (include/glint_cells.h:4-24 and
 * cuda/glint_encode.cu:17-34 / glint_codec.py:11-28 of Jadon-Fox/glint) written as
 * exact C99 hexadecimal float literals, so every compiler sees the same f32 bits.
 * Row h holds the 16 children of parent h in ascending order; concatenated rows
 * are strictly ascending over all 256 entries.  The table is data that must be
 * bit-identical to the reference's: tests/test_oracle.py pins it against
 * tests/golden/tables.json, which tests/golden/make_golden.py wrote from the
 * reference's own glint_codec.CELLS / PARENT.  The *_INIT macros let device
 * code define its own copies (host-side static arrays are not visible to
 * kernels).
 */
#ifndef GLINT_CELLS_H_
#define GLINT_CELLS_H_
#define GLINT_CELLS_INIT { \
    {-0x1.fb3d6ep-1f, -0x1.f2c25ep-1f, -0x1.eb5b1cp-1f, -0x1.e4c692p-1f, -0x1.ded87cp-1f, -0x1.d97160p-1f, -0x1.d47a02p-1f, -0x1.cfe0bep-1f, -0x1.cb97dcp-1f, -0x1.c79478p-1f, -0x1.c3cdcap-1f, -0x1.c03c9cp-1f, -0x1.bcdaf8p-1f, -0x1.b9a3dap-1f, -0x1.b69302p-1f, -0x1.b3a4ccp-1f}, \
    {-0x1.a94fa6p-1f, -0x1.9a5754p-1f, -0x1.8dfd0ap-1f, -0x1.836ca8p-1f, -0x1.7a2a1ep-1f, -0x1.71e664p-1f, -0x1.6a6bdep-1f, -0x1.639480p-1f, -0x1.5d443ep-1f, -0x1.5765d2p-1f, -0x1.51e8aep-1f, -0x1.4cbd86p-1f, -0x1.47de64p-1f, -0x1.43401ap-1f, -0x1.3edb76p-1f, -0x1.3aaa70p-1f}, \
    {-0x1.351b1cp-1f, -0x1.2e6980p-1f, -0x1.282750p-1f, -0x1.224506p-1f, -0x1.1cb632p-1f, -0x1.1770b6p-1f, -0x1.126c36p-1f, -0x1.0da1b4p-1f, -0x1.090b4cp-1f, -0x1.04a3f6p-1f, -0x1.006760p-1f, -0x1.f8a396p-2f, -0x1.f0bfe4p-2f, -0x1.e91deep-2f, -0x1.e1b8a6p-2f, -0x1.da8b8cp-2f}, \
    {-0x1.d23604p-2f, -0x1.c8d584p-2f, -0x1.bfca2ap-2f, -0x1.b70c9cp-2f, -0x1.ae966cp-2f, -0x1.a661f0p-2f, -0x1.9e6a22p-2f, -0x1.96aa90p-2f, -0x1.8f1f3ap-2f, -0x1.87c490p-2f, -0x1.809754p-2f, -0x1.7994a0p-2f, -0x1.72b9ccp-2f, -0x1.6c046ep-2f, -0x1.657252p-2f, -0x1.5f0176p-2f}, \
    {-0x1.57f578p-2f, -0x1.5057dap-2f, -0x1.48e430p-2f, -0x1.4197d2p-2f, -0x1.3a705cp-2f, -0x1.336b98p-2f, -0x1.2c8782p-2f, -0x1.25c23ap-2f, -0x1.1f1a0cp-2f, -0x1.188d5ep-2f, -0x1.121abap-2f, -0x1.0bc0c2p-2f, -0x1.057e2ep-2f, -0x1.fea39ep-3f, -0x1.f27512p-3f, -0x1.e66ea2p-3f}, \
    {-0x1.d9bbd6p-3f, -0x1.cc62bcp-3f, -0x1.bf361ep-3f, -0x1.b2339ap-3f, -0x1.a558fcp-3f, -0x1.98a42cp-3f, -0x1.8c1334p-3f, -0x1.7fa43ap-3f, -0x1.735582p-3f, -0x1.672564p-3f, -0x1.5b124ep-3f, -0x1.4f1ac6p-3f, -0x1.433d60p-3f, -0x1.3778c6p-3f, -0x1.2bcbb0p-3f, -0x1.2034e2p-3f}, \
    {-0x1.14456cp-3f, -0x1.07fe70p-3f, -0x1.f79a56p-4f, -0x1.df60a6p-4f, -0x1.c74d5ep-4f, -0x1.af5e1cp-4f, -0x1.97909cp-4f, -0x1.7fe2a8p-4f, -0x1.685220p-4f, -0x1.50dcf2p-4f, -0x1.39811ep-4f, -0x1.223cb2p-4f, -0x1.0b0dc4p-4f, -0x1.e7e4fcp-5f, -0x1.b9d218p-5f, -0x1.8bdf52p-5f}, \
    {-0x1.5ef7e2p-5f, -0x1.3316f2p-5f, -0x1.074a44p-5f, -0x1.b71dd2p-6f, -0x1.5fc3e6p-6f, -0x1.0880fcp-6f, -0x1.629eb6p-7f, -0x1.68a524p-8f, -0x1.848c0ap-13f, 0x1.505b9ap-8f, 0x1.5678c0p-7f, 0x1.026d04p-6f, 0x1.59ae88p-6f, 0x1.b106aap-6f, 0x1.043d98p-5f, 0x1.3008f8p-5f}, \
    {0x1.5a14bap-5f, 0x1.8260ecp-5f, 0x1.aac2b6p-5f, 0x1.d33c72p-5f, 0x1.fbd088p-5f, 0x1.1240b4p-4f, 0x1.26a8c6p-4f, 0x1.3b21c2p-4f, 0x1.4facf0p-4f, 0x1.644ba6p-4f, 0x1.78ff40p-4f, 0x1.8dc922p-4f, 0x1.a2aabap-4f, 0x1.b7a584p-4f, 0x1.ccbb02p-4f, 0x1.e1ecc8p-4f}, \
    {0x1.f6ab18p-4f, 0x1.057a8ep-3f, 0x1.0fae6ep-3f, 0x1.19f1f0p-3f, 0x1.2445dep-3f, 0x1.2eab06p-3f, 0x1.392246p-3f, 0x1.43ac80p-3f, 0x1.4e4aa0p-3f, 0x1.58fd9ep-3f, 0x1.63c678p-3f, 0x1.6ea640p-3f, 0x1.799e0cp-3f, 0x1.84af06p-3f, 0x1.8fda66p-3f, 0x1.9b2170p-3f}, \
    {0x1.a5fe5ap-3f, 0x1.b06e78p-3f, 0x1.baf8b6p-3f, 0x1.c59e44p-3f, 0x1.d0605ep-3f, 0x1.db4050p-3f, 0x1.e63f7ap-3f, 0x1.f15f52p-3f, 0x1.fca162p-3f, 0x1.0403a6p-2f, 0x1.09c968p-2f, 0x1.0fa2e2p-2f, 0x1.159112p-2f, 0x1.1b9504p-2f, 0x1.21afd8p-2f, 0x1.27e2c2p-2f}, \
    {0x1.2dbe2ap-2f, 0x1.333e22p-2f, 0x1.38d2d4p-2f, 0x1.3e7d42p-2f, 0x1.443e82p-2f, 0x1.4a17bcp-2f, 0x1.500a32p-2f, 0x1.56173cp-2f, 0x1.5c404ap-2f, 0x1.6286eep-2f, 0x1.68ecdap-2f, 0x1.6f73e8p-2f, 0x1.761e16p-2f, 0x1.7ced96p-2f, 0x1.83e4cap-2f, 0x1.8b0658p-2f}, \
    {0x1.9197b0p-2f, 0x1.978e92p-2f, 0x1.9da5fcp-2f, 0x1.a3dfe0p-2f, 0x1.aa3e5cp-2f, 0x1.b0c3bep-2f, 0x1.b77292p-2f, 0x1.be4da4p-2f, 0x1.c5580ep-2f, 0x1.cc953ep-2f, 0x1.d4090ap-2f, 0x1.dbb7b8p-2f, 0x1.e3a61ap-2f, 0x1.ebd9a0p-2f, 0x1.f45874p-2f, 0x1.fd29a6p-2f}, \
    {0x1.027dccp-1f, 0x1.05d898p-1f, 0x1.094e1ap-1f, 0x1.0ce06cp-1f, 0x1.1091eap-1f, 0x1.146544p-1f, 0x1.185d82p-1f, 0x1.1c7e22p-1f, 0x1.20cb26p-1f, 0x1.25493ap-1f, 0x1.29fdccp-1f, 0x1.2eef4ep-1f, 0x1.34256cp-1f, 0x1.39a96cp-1f, 0x1.3f869ep-1f, 0x1.45cb14p-1f}, \
    {0x1.4b027cp-1f, 0x1.4ef5c4p-1f, 0x1.531bc2p-1f, 0x1.57751cp-1f, 0x1.5c0aaep-1f, 0x1.60e44ap-1f, 0x1.660b74p-1f, 0x1.6b8be4p-1f, 0x1.71743ep-1f, 0x1.77d738p-1f, 0x1.7ecd32p-1f, 0x1.8676d8p-1f, 0x1.8f0174p-1f, 0x1.98ae78p-1f, 0x1.a3e1d2p-1f, 0x1.b13fdcp-1f}, \
    {0x1.ba6bb0p-1f, 0x1.bd3180p-1f, 0x1.c016bcp-1f, 0x1.c31e88p-1f, 0x1.c64c8cp-1f, 0x1.c9a50ep-1f, 0x1.cd2d18p-1f, 0x1.d0eab4p-1f, 0x1.d4e528p-1f, 0x1.d92552p-1f, 0x1.ddb642p-1f, 0x1.e2a5e4p-1f, 0x1.e80630p-1f, 0x1.edeee0p-1f, 0x1.f48044p-1f, 0x1.fbe7f2p-1f}, \
}
static const float GLINT_CELLS[16][16] = GLINT_CELLS_INIT;
/* Parent (hole) centres; GLINT_PARENT[7] == 0. */
#define GLINT_PARENT_INIT { -0x1.000000p+0f, -0x1.647362p-1f, -0x1.0cd660p-1f, -0x1.946540p-2f, -0x1.23449ap-2f, -0x1.7a6a7ep-3f, -0x1.74f0e2p-4f, 0x0.0p+0f, 0x1.45f5fep-4f, 0x1.4995c6p-3f, 0x1.f809bap-3f, 0x1.5a0674p-2f, 0x1.c34970p-2f, 0x1.200f56p-1f, 0x1.722766p-1f, 0x1.000000p+0f }
static const float GLINT_PARENT[16] = GLINT_PARENT_INIT;
#ifndef P7_CELLS
#define P7_CELLS GLINT_CELLS
#endif
#endif
