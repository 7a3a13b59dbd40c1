from teamredbench_b200.profiling.registry import (  # noqa: F401
    ProfilingEngineDefinition,
    ProfilingLaunch,
    get_profile_engine,
    list_profile_engines,
    register_profile_engine,
)
