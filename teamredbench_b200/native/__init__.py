from teamredbench_b200.native.registry import (  # noqa: F401
    NativeKernelDefinition,
    get_native_kernel,
    list_native_kernels,
    register_native_kernel,
)
