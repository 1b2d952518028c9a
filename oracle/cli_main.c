/*
 * The reference's command-line program (atlas_dynamic_infer: argv contract,
 * stdout text, stop tokens, exit codes - src/brain_runtime.c:1921-2064),
 * built on Linux from src/brain_runtime.c compiled in place behind the Win32
 * shim. oracle/Makefile links it twice: against the CPU stub of the device
 * plugin (the reference's own CPU path) and against libatlas_cuda.so, whose
 * brain_gpu_* entry points replace the Direct3D 12 plugin (src/gpu_matvec.h)
 * - the drop-in the plugin ABI exists for. tests/test_gpu_boundary.py runs
 * both on a synthetic model and compares their output.
 */
#include "brain_runtime.c"

int main(int argc, char **argv) { return run_main_utf8(argc, argv); }
