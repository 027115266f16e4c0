"""the whole persistence stack (region, event log, registry,
graph analysis, JSON + .cugraph archive, manifest, template/on-demand restore,
fault handling) on the CPU mock driver, SAVE and LOAD in separate processes."""

import json
import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
MOCK = os.path.join(ROOT, "foundry_b200", "lib", "libfoundry_mockcuda.so")


def _run(*args, timeout=300):
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=MOCK, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    res = subprocess.run([sys.executable, os.path.join(HERE, "mock_scenarios.py"), *args], env=env,
                         capture_output=True, text=True, timeout=timeout)
    assert res.returncode == 0, f"scenario {args[0]} failed:\n{res.stdout}\n{res.stderr}"
    return res.stdout


@pytest.fixture(scope="module")
def saved(tmp_path_factory):
    wd = str(tmp_path_factory.mktemp("mock_archive"))
    out = _run("save", wd)
    assert "SAVE OK" in out
    return wd


def test_archive_layout(saved):
    a = os.path.join(saved, "archive")
    files = set(os.listdir(a))
    assert {"graph_manifest.json", "fatbin_image_packed.img", "fatbin_entrypoint_packed.txt"} <= files
    assert sum(f.endswith(".cugraph") for f in files) == 64
    m = json.load(open(os.path.join(a, "graph_manifest.json")))
    assert len(m["topology_groups"]) == 4
    assert sum(len(g["members"]) for g in m["topology_groups"]) == 64
    # on-demand members lose their dependency table in JSON (binary keeps it)
    tmpl = {g["template"] for g in m["topology_groups"]}
    for g in m["topology_groups"]:
        for f in g["members"]:
            has = "dependencies" in json.load(open(os.path.join(a, f)))
            assert has == (f in tmpl)
    # pack: [u64 hash][u64 size][bytes]; the 1 MB image plus its header
    img = open(os.path.join(a, "fatbin_image_packed.img"), "rb").read()
    size = int.from_bytes(img[8:16], "little")
    assert size > (1 << 20) and len(img) == 16 + size
    txt = open(os.path.join(a, "fatbin_entrypoint_packed.txt")).read().splitlines()
    assert txt[1].startswith("cuLibraryLoadData") and txt[2] == "10" and txt[-1] == "---"


def test_load_round_trip(saved):
    out = _run("load", saved)
    assert "LOAD OK 64 4" in out


def test_numeric_save_load_bit_exact(saved):
    _run("numeric", saved, "save")
    _run("numeric", saved, "load")
    a = json.load(open(os.path.join(saved, "num_save.json")))
    b = json.load(open(os.path.join(saved, "num_load.json")))
    assert a == b
    # y = 1 + 2 launches * (0.25+0.5+...+1.5) * x
    assert a[1] == pytest.approx(1 + 2 * 5.25 * 0.5 * 97)


def test_programmatic_dependency_edges_round_trip(tmp_path):
    """Graphs captured with programmatic dependent launch (vLLM's and
    FlashInfer's kernels use it) carry edge data that the plain edge query
    cannot return; it is persisted and restored."""
    assert "PDL OK" in _run("pdl", str(tmp_path))


def test_generator_records_and_relocation(saved):
    assert "RNG OK" in _run("rng", saved)


def test_fault_injection(saved):
    assert "FAULTS OK" in _run("faults", saved)


def test_cluster_launch_dims_round_trip(tmp_path):
    """Kernel nodes launched in thread-block clusters (the two-SM GEMM's shape)
    keep their cluster dims through analysis, JSON, .cugraph and restore, and
    only graphs with the same cluster shapes share a topology template."""
    wd = str(tmp_path)
    assert "CLUSTER SAVE OK" in _run("cluster", wd, "save")
    assert "CLUSTER LOAD OK" in _run("cluster", wd, "load")


def test_memcpy_event_empty_nodes_round_trip(tmp_path):
    """Every node type of the graph store (kernel, memcpy, memset, event
    record / wait, empty) through analysis, JSON, .cugraph and restore."""
    wd = str(tmp_path)
    assert "MIXED SAVE OK" in _run("mixed", wd, "save")
    assert "MIXED LOAD OK" in _run("mixed", wd, "load")


def test_manifest_refuses_graphs_without_topology_key(tmp_path):
    """A graph without a topology key cannot join a group: writing a manifest
    that silently leaves it out would hide that, so the call raises."""
    from foundry_b200.graphs import save_graph_manifest

    (tmp_path / "graph_0.json").write_text(json.dumps({"topology_key": "k", "nodes": [], "dependencies": []}))
    (tmp_path / "graph_1.json").write_text(json.dumps({"nodes": []}))
    with pytest.raises(ValueError, match="topology_key"):
        save_graph_manifest(str(tmp_path))
    assert not (tmp_path / "graph_manifest.json").exists()
    (tmp_path / "graph_1.json").write_text(json.dumps({"topology_key": "k", "nodes": [], "dependencies": [1]}))
    (tmp_path / "graph_10.json").write_text(json.dumps({"topology_key": "j", "nodes": []}))
    m = save_graph_manifest(str(tmp_path))
    assert m["topology_groups"] == [
        {"topology_key": "k", "template": "graph_0.json", "members": ["graph_0.json", "graph_1.json"]},
        {"topology_key": "j", "template": "graph_10.json", "members": ["graph_10.json"]}]
    assert "dependencies" in json.loads((tmp_path / "graph_0.json").read_text())
    assert "dependencies" not in json.loads((tmp_path / "graph_1.json").read_text())
