// Oracle (test infrastructure only): the benchmark workloads of
// minitensor_cpp_b200/host/workloads.cpp compiled against the UNMODIFIED
// reference, CPU device only.  Both sides therefore run the same graphs; this
// copy is the CPU baseline and the loss-curve reference.
#define MTB_CPU_ONLY 1
#include "workloads.cpp"
