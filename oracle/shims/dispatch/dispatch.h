/*
 * Linux stand-in for <dispatch/dispatch.h>.  TEST INFRASTRUCTURE ONLY.
 * oracle/build_ref.py rewrites every dispatch_apply block into an OpenMP
 * parallel-for and every dispatch_async block into an inline block before
 * compiling, so no libdispatch symbol is referenced; this header only has to
 * exist.
 */
#ifndef SS_ORACLE_SHIM_DISPATCH_H
#define SS_ORACLE_SHIM_DISPATCH_H
#endif
