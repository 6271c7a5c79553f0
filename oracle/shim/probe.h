/*
 * probe.h — force-included (g++ -include) into an unchanged akili-bench
 * benchmarks/<bench>/main.cpp when oracle/build_oracle.py builds the oracle pin
 * and golden-vector capture binaries.  TEST INFRASTRUCTURE.
 *
 * In the reference harnesses `fabsf` / `std::fabs` appear only in the verify
 * loops (diff = fabsf(actual - expected), rel = diff / fabsf(expected), and
 * flash's Comparator::compare), and integer `std::abs` only in the kb2 ulp
 * checks (std::abs(actual_bits - expected_bits)); both are redirected.  Redirecting them gives two modes, chosen by
 * the AKILI_PROBE environment variable:
 *
 *   exact   |x| is reported as 0 when x == 0 and as 1e30 otherwise, so every
 *           element whose device value is not bit-identical to the
 *           reference gold counts as an error under any of the harness
 *           tolerances, and the harness prints PASSED! only on exact
 *           equality (+0 and -0 compare equal).
 *   record  |x| is computed normally and every argument x is appended, as
 *           raw fp32, to the file named by AKILI_PROBE_FILE.  With a device
 *           that leaves the output at 0, x = 0 - expected, which exposes the
 *           reference gold values exactly (sign included).
 *
 * Unset: plain fabs.
 */
#ifndef AKILI_PROBE_H_
#define AKILI_PROBE_H_

/* Pull in everything the harnesses include before the macros exist. */
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <iostream>
#include <string.h>
#include <unistd.h>
#include <vector>

float akili_probe_fabsf(float x);
int akili_probe_iabs(int x);

#define fabsf akili_probe_fabsf
namespace std {
inline float akili_probe_fabs(float x) { return ::akili_probe_fabsf(x); }
}  // namespace std
#define fabs akili_probe_fabs
/* The kb2 harnesses compare results in ulps: std::abs(fa.i - fb.i). */
namespace std {
inline int akili_probe_abs(int x) { return ::akili_probe_iabs(x); }
}  // namespace std
#define abs akili_probe_abs

#endif
