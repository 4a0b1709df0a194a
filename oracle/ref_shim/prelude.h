/* Force-included before the reference headers when the reference kernels are
 * compiled on Linux (oracle/build_ref.sh). glibc >= 2.38 declares the C23
 * functions fmaximum/fminimum, which collide with the reference's float
 * constants of the same names; renaming them here keeps every use consistent.
 * <atomic> is included because ca.cu uses std::atomic without including it.
 * TEST INFRASTRUCTURE ONLY. */
#pragma once
#include <cmath>
#include <cstdio>
#include <atomic>
#define fmaximum aic_ref_fmaximum
#define fminimum aic_ref_fminimum
namespace std { using ::sqrtf; }
