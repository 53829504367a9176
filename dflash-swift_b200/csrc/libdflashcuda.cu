// Single translation unit of libdflashcuda.so (keeps one copy of the device error
// word and lets the compiler see every kernel of the library at once).
#include "abi.cu"
#include "qmm.cu"
#include "gdn.cu"
#include "tp.cu"
#include "stack.cu"
#include "stack_driver.cu"
