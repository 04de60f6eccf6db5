"""Link-level drop-in check (CPU only, no kernel ever runs).

The reference links its kernels as a static archive (anima_kernels, CMakeLists.txt:30-48)
into the executable. tests/integration/caller.cpp stands in for transformer.cpp: it
declares rms_norm_bf16 as kernels.h does and calls it. Linked against

  * the reference archive as built + libanima_b200.so: the archive's own definition is
    part of the executable and wins, so the B200 library is NOT used (status 0);
  * the archive after anima.cu_b200/integrate/localize_reference_launchers.sh +
    libanima_b200.so: the call binds to the B200 shim (status -2, BAD_SHAPE for the
    N = 0, D = 0 probe).

The probe is safe anywhere: the reference's launcher gets a zero-size grid and launches
nothing, the B200 shim rejects the shape before touching the GPU.
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "anima.cu_b200")
ARCHIVE = os.path.join(ROOT, "oracle", "_ref", "libref_kernels.a")
SCRIPT = os.path.join(PKG, "integrate", "localize_reference_launchers.sh")
CALLER = os.path.join(ROOT, "tests", "integration", "caller.cpp")


def _nm_globals(path):
    out = subprocess.run(["nm", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if len(line.split()) == 3 and line.split()[1] == "T"}


def test_replaced_launcher_list_matches_the_library():
    import anima_b200
    import refkernels

    listed = [l.strip() for l in open(os.path.join(PKG, "integrate", "replaced_launchers.txt"))
              if l.strip() and not l.startswith("#")]
    assert sorted(listed) == sorted(m for m, _ in refkernels.LAUNCHERS.values())
    out = subprocess.run(["nm", "-D", "--defined-only", anima_b200.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines()}
    assert set(listed) <= exported


@pytest.fixture(scope="module")
def archives(tmp_path_factory):
    if not os.path.exists(ARCHIVE):
        pytest.skip("oracle/_ref/libref_kernels.a not built (make -C oracle ref-static needs the reference tree)")
    if shutil.which("nvcc") is None or shutil.which("objcopy") is None:
        pytest.skip("nvcc/objcopy not available")
    d = tmp_path_factory.mktemp("link")
    plain = str(d / "libref_plain.a")
    local = str(d / "libref_local.a")
    shutil.copy(ARCHIVE, plain)
    subprocess.run([SCRIPT, plain, local], check=True)
    return d, plain, local


def test_localization_hides_exactly_the_replaced_launchers(archives):
    _, plain, local = archives
    replaced = {l.strip() for l in open(os.path.join(PKG, "integrate", "replaced_launchers.txt"))
                if l.strip() and not l.startswith("#")}
    g_plain, g_local = _nm_globals(plain), _nm_globals(local)
    assert replaced <= g_plain
    assert not (replaced & g_local)
    # everything else the reference archive defines stays available to its callers
    assert g_plain - replaced == g_local


def _link_and_run(d, archive, name):
    exe = str(d / name)
    subprocess.run(["nvcc", "-std=c++17", "-o", exe, CALLER, archive, f"-L{PKG}", "-lanima_b200",
                    f"-Xlinker=-rpath={PKG}"], check=True, capture_output=True)
    return int(subprocess.run([exe], capture_output=True, text=True, check=True).stdout.strip())


def test_reference_archive_as_built_shadows_the_library(archives):
    d, plain, _ = archives
    assert _link_and_run(d, plain, "caller_plain") == 0


def test_localized_archive_binds_callers_to_the_b200_library(archives):
    d, _, local = archives
    assert _link_and_run(d, local, "caller_local") == -2


CALLERS = ("transformer", "qwen3", "llm_adapter", "vae")


def test_reference_callers_resolve_every_launcher(archives):
    """The reference's own callers (transformer.cpp, qwen3.cpp, llm_adapter.cpp, vae.cpp,
    compiled unchanged into oracle/_ref/callers by `make -C oracle callers`): every
    kernels.h launcher they leave undefined must be one this library replaces, defined by
    libanima_b200.so and hidden in the localized reference archive, so each binds to it."""
    import anima_b200

    objs = {c: os.path.join(ROOT, "oracle", "_ref", "callers", c + ".o") for c in CALLERS}
    if not all(os.path.exists(o) for o in objs.values()):
        pytest.skip("oracle/_ref/callers not built (make -C oracle callers needs the reference tree)")
    _, plain, local = archives
    out = subprocess.run(["nm", "-D", "--defined-only", anima_b200.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    lib = {line.split()[-1] for line in out.splitlines() if " T " in line}
    g_plain, g_local = _nm_globals(plain), _nm_globals(local)
    replaced = {l.strip() for l in open(os.path.join(PKG, "integrate", "replaced_launchers.txt"))
                if l.strip() and not l.startswith("#")}
    bound = 0
    for name, obj in objs.items():
        und = set(subprocess.run(["nm", "-u", obj], capture_output=True, text=True, check=True).stdout.split())
        launchers = und & (g_plain | replaced)
        assert launchers, f"{name}.cpp calls no reference launcher?"
        unresolved = [s for s in launchers if s not in lib and s not in g_local]
        assert not unresolved, f"{name}.cpp: unresolved launchers {unresolved}"
        kept = sorted(launchers - replaced)
        assert not kept, f"{name}.cpp: launchers left to the reference: {kept}"
        for s in launchers:
            assert s in lib and s not in g_local, f"{name}.cpp: {s} would not bind to the B200 library"
        bound += len(launchers)
    assert bound == 38  # 13 + 11 + 8 + 6 launcher references across the four callers
