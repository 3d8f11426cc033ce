/* Empty stand-in for <mkl.h>.  The reference's src/general.cuh:6 includes
 * <mkl.h> but calls nothing from it; MKL is not installed here, so the
 * reference's host sources are compiled against this empty header. */
#ifndef TCASPMM_ORACLE_MKL_STUB_H
#define TCASPMM_ORACLE_MKL_STUB_H
#endif
