"""runtime: the cuda target's launch-list lowering (program) and its ctypes binding (cuda)."""
