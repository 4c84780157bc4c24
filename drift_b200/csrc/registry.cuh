// The by-name kernel table: what drift_module_get_function looks names up in
// when given no module, as the runner's KernelModule.function looks a name up
// in a loaded code object (runner/src/drift/runner/native/KernelModule.scala:26-27).
// Each kernel file registers its launchable kernels at load time.
#pragma once

namespace drift {

struct KernelEntry {
  const char* name;
  const void* function;  // what cudaLaunchKernel takes
};

// Adds a kernel; returns its index. Called from static initialisers only.
int register_kernel(const char* name, const void* function);
int kernel_count();
const KernelEntry* kernel_at(int index);
const KernelEntry* find_kernel(const char* name);

}  // namespace drift

#define DRIFT_REGISTER_CAT2(a, b) a##b
#define DRIFT_REGISTER_CAT(a, b) DRIFT_REGISTER_CAT2(a, b)
#define DRIFT_REGISTER(name, function)                                              \
  static const int DRIFT_REGISTER_CAT(drift_registered_, __COUNTER__) =              \
      ::drift::register_kernel(#name, reinterpret_cast<const void*>(&function));
