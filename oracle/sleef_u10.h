/* Portable restatement of SLEEF 3.7 u10 float exp/sin/cos (oracle only).
 * TEST INFRASTRUCTURE: used by the CPU oracle and the oracle/_ref build. */
#ifndef ORACLE_SLEEF_U10_H
#define ORACLE_SLEEF_U10_H

/* One lane of Sleef_expf4_u10 (speech-mac vendor/sleef/sleefinline_advsimd.h:5589). */
float oracle_sleef_expf(float d);
/* Sleef_expf4_u10 on four lanes, in place. */
void oracle_sleef_expf4(float values[4]);
/* Sleef_cosf4_u10 / Sleef_sinf4_u10 on one four-lane vector, keeping the
 * vector-wide choice between the Cody-Waite and rempif reductions. */
void oracle_sleef_sincosf4(const float d[4], float cosines[4], float sines[4]);

#endif
