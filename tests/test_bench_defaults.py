"""bench.py's decode-step fusion defaults (host logic, no GPU): config 4 fuses the row-parallel GEMVs with their
allreduce at two ranks only, where that measured faster; from four ranks on, separate kernels measured faster."""
import argparse

import bench


def args(**kw):
    return argparse.Namespace(**kw)


def test_config4_fuses_gemv_allreduce_at_two_ranks_only():
    assert bench.fuse_arg(args(), 4, 2) == ("epilogue", "gemv_allreduce")
    for world in (1, 4, 8):
        assert bench.fuse_arg(args(), 4, world) == ("epilogue",)


def test_explicit_fuse_wins_and_config3_default_is_unfused():
    assert bench.fuse_arg(args(fuse="epilogue,gemv_allreduce"), 4, 8) == ("epilogue", "gemv_allreduce")
    assert bench.fuse_arg(args(fuse=""), 4, 2) == ()
    assert bench.fuse_arg(args(), 3) == ()
