/*
 * ref_shim.c -- exports the reference's own plain-C block decoder
 * (lxdde/ports/nouveau/q4k_decode.h of demonodojo/soso) as a shared library,
 * so the tests can check oracle.c against the reference's code itself.
 *
 * TEST INFRASTRUCTURE ONLY.  The header is NOT copied into this repository:
 * oracle/Makefile compiles this shim with -I pointing at the reference
 * checkout, and the result lands in oracle/_ref/ (git-ignored).
 */
#include "q4k_decode.h"

#define REF_API __attribute__((visibility("default")))

REF_API float ref_q4k_f16(unsigned short bits) { return q4k_f16(bits); }
REF_API void ref_q4k_scale_min(const unsigned char *s, int j, unsigned char *sc, unsigned char *m)
{
    q4k_scale_min(s, j, sc, m);
}
REF_API float ref_q4k_dot_sub(const unsigned char *blk, int j, const float *x) { return q4k_dot_sub(blk, j, x); }
REF_API float ref_q4k_dot_block(const unsigned char *blk, const float *x) { return q4k_dot_block(blk, x); }
REF_API float ref_q80_dot_block(const unsigned char *blk, const float *x) { return q80_dot_block(blk, x); }
