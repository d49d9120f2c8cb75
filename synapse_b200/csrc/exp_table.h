/* 2^(j/64) for j = 0..63, each split into a float and the float nearest the
 * remainder (from the double 2^(j/64)): the table of the library's expf
 * (Tang's method), shared by the device code (common.cuh) and the host-side
 * scan that finds where the C runtime's expf rounds differently
 * (libm_expf_scan.c). Plain C: both nvcc and gcc include it. */
#ifndef SYN_EXP_TABLE_H
#define SYN_EXP_TABLE_H
#define SYN_EXP2_J64_TABLE \
    {0x1.p+0f, 0.0f}, {0x1.02c9a4p+0f, -0x1.887fa0p-28f}, \
    {0x1.059b0ep+0f, -0x1.9d4f52p-25f}, {0x1.087452p+0f, -0x1.e2990ep-26f}, \
    {0x1.0b5586p+0f, 0x1.9f3122p-25f}, {0x1.0e3ec4p+0f, -0x1.a585ccp-25f}, \
    {0x1.11301ep+0f, -0x1.fdb496p-25f}, {0x1.1429aap+0f, 0x1.d525bcp-25f}, \
    {0x1.172b84p+0f, -0x1.c15742p-27f}, {0x1.1a35bep+0f, 0x1.6df96ep-25f}, \
    {0x1.1d4874p+0f, -0x1.d2e8cap-25f}, {0x1.2063b8p+0f, 0x1.0c519ap-25f}, \
    {0x1.2387a6p+0f, 0x1.ceac48p-25f}, {0x1.26b456p+0f, 0x1.789f38p-26f}, \
    {0x1.29e9e0p+0f, -0x1.5c0424p-25f}, {0x1.2d285ap+0f, 0x1.b900c2p-26f}, \
    {0x1.306fe0p+0f, 0x1.4636e2p-25f}, {0x1.33c08cp+0f, -0x1.b37d20p-25f}, \
    {0x1.371a74p+0f, -0x1.18aac6p-25f}, {0x1.3a7db4p+0f, -0x1.634c02p-25f}, \
    {0x1.3dea64p+0f, 0x1.824684p-25f}, {0x1.4160a2p+0f, 0x1.f72e2ap-28f}, \
    {0x1.44e086p+0f, 0x1.8624b4p-30f}, {0x1.486a2cp+0f, -0x1.47d866p-25f}, \
    {0x1.4bfdaep+0f, -0x1.593abcp-25f}, {0x1.4f9b28p+0f, -0x1.2c5a6cp-25f}, \
    {0x1.5342b6p+0f, -0x1.2c5610p-25f}, {0x1.56f474p+0f, -0x1.295b04p-25f}, \
    {0x1.5ab07ep+0f, -0x1.5bd5ecp-27f}, {0x1.5e76f2p+0f, -0x1.4a5bd8p-25f}, \
    {0x1.6247ecp+0f, -0x1.f8b550p-25f}, {0x1.662388p+0f, 0x1.2a9112p-27f}, \
    {0x1.6a09e6p+0f, 0x1.9fcef4p-26f}, {0x1.6dfb24p+0f, -0x1.cd72e8p-27f}, \
    {0x1.71f75ep+0f, 0x1.1d8beep-25f}, {0x1.75feb6p+0f, -0x1.37b306p-25f}, \
    {0x1.7a1148p+0f, -0x1.829fd0p-25f}, {0x1.7e2f34p+0f, -0x1.261634p-25f}, \
    {0x1.82589ap+0f, -0x1.accc7cp-26f}, {0x1.868d9ap+0f, -0x1.2edb44p-26f}, \
    {0x1.8ace54p+0f, 0x1.15506ep-27f}, {0x1.8f1aeap+0f, -0x1.baa232p-26f}, \
    {0x1.93737cp+0f, -0x1.e64744p-25f}, {0x1.97d82ap+0f, -0x1.0d8d80p-31f}, \
    {0x1.9c4918p+0f, 0x1.51f848p-27f}, {0x1.a0c668p+0f, -0x1.2886a6p-26f}, \
    {0x1.a5503cp+0f, -0x1.b83b54p-25f}, {0x1.a9e6b6p+0f, -0x1.50c048p-25f}, \
    {0x1.ae89fap+0f, -0x1.a94b14p-26f}, {0x1.b33a2cp+0f, -0x1.ec3a82p-26f}, \
    {0x1.b7f770p+0f, -0x1.a09438p-25f}, {0x1.bcc1eap+0f, -0x1.f687c6p-25f}, \
    {0x1.c199bep+0f, -0x1.3d56b2p-27f}, {0x1.c67f12p+0f, 0x1.cafa2ap-25f}, \
    {0x1.cb720ep+0f, -0x1.8837ccp-27f}, {0x1.d072d4p+0f, 0x1.40f130p-25f}, \
    {0x1.d5818ep+0f, -0x1.822dbcp-27f}, {0x1.da9e60p+0f, 0x1.ed9942p-27f}, \
    {0x1.dfc974p+0f, -0x1.908c94p-25f}, {0x1.e502eep+0f, 0x1.e2cffep-26f}, \
    {0x1.ea4afap+0f, 0x1.52486cp-27f}, {0x1.efa1bep+0f, 0x1.cc2b44p-25f}, \
    {0x1.f50766p+0f, -0x1.246eb0p-26f}, {0x1.fa7c18p+0f, 0x1.9e90d8p-28f}
#endif
