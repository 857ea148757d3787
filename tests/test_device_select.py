"""Local-rank device binding (C++), tested without a GPU via fake device counts."""
import pytest

from multi_gpu_flashattention_b200.utils.device import choose_device, local_rank

VARS = ["OMPI_COMM_WORLD_LOCAL_RANK", "MV2_COMM_WORLD_LOCAL_RANK", "SLURM_LOCALID",
        "MPI_LOCALRANKID", "PMI_LOCAL_RANK", "PALS_LOCAL_RANK", "LOCAL_RANK"]


@pytest.fixture
def clean_env(monkeypatch):
    for v in VARS + ["ALLOW_GPU_OVERSUBSCRIBE"]:
        monkeypatch.delenv(v, raising=False)
    return monkeypatch


def test_precedence(clean_env):
    clean_env.setenv("LOCAL_RANK", "3")
    clean_env.setenv("SLURM_LOCALID", "1")
    assert local_rank() == (1, "SLURM_LOCALID")
    clean_env.setenv("OMPI_COMM_WORLD_LOCAL_RANK", "2")
    assert local_rank() == (2, "OMPI_COMM_WORLD_LOCAL_RANK")


def test_fallback_and_oversubscribe(clean_env):
    dev, lr, src, err = choose_device(8, 5)
    assert (dev, lr, src, err) == (5, 5, "fallback", "")
    clean_env.setenv("LOCAL_RANK", "9")
    dev, lr, src, err = choose_device(8, 0)
    assert dev == -1 and "ALLOW_GPU_OVERSUBSCRIBE" in err
    clean_env.setenv("ALLOW_GPU_OVERSUBSCRIBE", "1")
    dev, lr, src, err = choose_device(8, 0)
    assert dev == 1 and err == ""


def test_no_devices(clean_env):
    dev, _, _, err = choose_device(0, 0)
    assert dev == -1 and "No CUDA devices" in err


def test_product_build_is_not_the_debug_build():
    """The in-tree extension is the normal build (MGFA_DEBUG adds bounds checks)."""
    import pytest
    try:
        from multi_gpu_flashattention_b200._ext import C
        m = C()
    except Exception as e:  # pragma: no cover - extension not built
        pytest.skip(f"extension not built: {e}")
    assert m.debug_build() is False
