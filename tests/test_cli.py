"""The reference-compatible CLI's argument handling (no GPU needed): fewer than the six
positional arguments print the usage line and fail (src/dist_spmm_node.cu:27-44); a
".mtx" file is refused as the reference's load_from_mtx stub does (src/sparse_matrix.h:68-81)."""
import os
import subprocess

from distspmm_b200 import build


def _exe():
    return os.path.join(build.BIN, "dist_spmm_node")


def test_usage_on_missing_arguments():
    r = subprocess.run([_exe()], capture_output=True, text=True, timeout=60)
    assert r.returncode != 0
    assert "Usage:" in r.stdout + r.stderr
    assert "<dims> <task_dist> <comm_type> <n_rolls> <repeat>" in r.stdout + r.stderr


def test_mtx_files_are_refused():
    r = subprocess.run([_exe(), "graph.mtx", "64", "2", "2", "2", "7"], capture_output=True, text=True, timeout=60)
    assert r.returncode != 0
    assert "mtx" in (r.stdout + r.stderr).lower()


def test_alias_binary_exists():
    assert os.path.exists(os.path.join(build.BIN, "dist_spmm"))
