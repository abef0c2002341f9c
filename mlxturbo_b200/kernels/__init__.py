"""Host-side mirror of mlxturbo/kernels/: same module names and entry points,
each backed by libmlxturbo_b200.so kernels for sm_100a."""
