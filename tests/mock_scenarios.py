"""CPU-only scenarios run against the mock driver (libfoundry_mockcuda.so).

Each scenario runs in its own process (the driver is chosen once per process),
started by tests/test_mock_archive.py:

    FOUNDRY_CUDA_DRIVER=.../libfoundry_mockcuda.so python tests/mock_scenarios.py <name> <workdir> [...]

Scenario "save" builds the BASELINE config-1 workload (200 region allocations
log-uniform 256 B..64 MB with seed 0, a 1 MB random code image, 64 graphs in 4
topology groups of 32-kernel chains with 8 seeded random args each) and writes
an archive; "load" restores it in a fresh process and checks everything
byte-for-byte against the SAVE process's record.
"""

from __future__ import annotations

import json
import os
import random
import struct
import sys

# FOUNDRY_TEST_REGION_BASE moves the region (ThreadSanitizer reserves the
# default 0x600000000000 range for itself)
BASE = int(os.environ.get("FOUNDRY_TEST_REGION_BASE", "0x600000000000"), 0)
REGION = 64 << 30
N_GRAPHS, N_GROUPS, CHAIN, N_ARGS = 64, 4, 32, 8
PARAM_SIZES = [8, 8, 8, 4, 4, 16, 8, 32]  # 8 args: pointers and seeded random bytes


def _core():
    # FOUNDRY_PKG_ROOT selects another build of the package (e.g. the
    # ThreadSanitizer build); default: this repository
    sys.path.insert(0, os.environ.get("FOUNDRY_PKG_ROOT") or os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import foundry_b200 as fb

    c = fb.core()
    assert c.driver_is_mock(), "scenarios must run on the mock driver"
    return fb, c


def _image_bytes(seed: int = 0) -> bytes:
    names = [f"fbmock_k{j}:{','.join(map(str, PARAM_SIZES))}" for j in range(8)]
    names += ["fbmock_axpy_f32:8,8,4,4", "fbmock_fill_u32:8,4,4"]
    header = ("FBMOCK\n" + "\n".join(names) + "\n\n").encode()
    rnd = random.Random(seed)
    return header + bytes(rnd.getrandbits(8) for _ in range(1 << 20))


def _alloc_sizes(seed: int = 0) -> list[int]:
    import math

    rnd = random.Random(seed)
    lo, hi = math.log(256), math.log(64 << 20)
    return [max(256, int(math.exp(rnd.uniform(lo, hi))) // 256 * 256) for _ in range(200)]


def _graph_json(gi: int, img_hash: int, ptrs: list[int]) -> str:
    """Graph gi: group g = gi % 4 has a memset at position 8*g (distinct node-type
    sequence per group); members differ in their random args and pointers."""
    g = gi % N_GROUPS
    rnd = random.Random(1000 + gi)
    nodes = []
    for n in range(CHAIN):
        if n == 8 * g:
            nodes.append({"id": n, "type": "MemsetNode", "params": {
                "dst": ptrs[rnd.randrange(len(ptrs))], "elementSize": 4, "height": 1, "pitch": 0,
                "value": rnd.getrandbits(32), "width": 64}})
            continue
        params = []
        off = 0
        for i, sz in enumerate(PARAM_SIZES):
            if sz == 8 and i < 3:
                val = struct.pack("<Q", ptrs[rnd.randrange(len(ptrs))] + 256 * rnd.randrange(4))
            else:
                val = bytes(rnd.getrandbits(8) for _ in range(sz))
            params.append({"index": i, "offset": off, "size": sz, "value_hex": val.hex()})
            off += sz
        nodes.append({"id": n, "type": "KernelNode", "params": {
            "blockDimX": 128, "blockDimY": 1, "blockDimZ": 1,
            "gridDimX": 1 + rnd.randrange(512), "gridDimY": 1, "gridDimZ": 1,
            "sharedMemBytes": 0, "kernelParams": params,
            "function_name": f"fbmock_k{(n + g) % 8}", "kernel_source_binary_hash": f"{img_hash:016x}",
            "func_attrs": {"max_dynamic_shared_size_bytes": 0, "preferred_shared_memory_carveout": -1,
                           "cluster_scheduling_policy_preference": 0, "required_cluster_width": 0,
                           "required_cluster_height": 0, "required_cluster_depth": 0}}})
    deps = [{"from": i, "to": i + 1} for i in range(CHAIN - 1)]
    return json.dumps({"nodes": nodes, "dependencies": deps, "topology_key": "", "generators": []})


def scenario_save(workdir: str) -> None:
    fb, c = _core()
    archive = os.path.join(workdir, "archive")
    os.makedirs(archive, exist_ok=True)
    c.set_allocation_region(BASE, REGION)
    # 1) region: 200 allocations, recorded as allocator events
    c.start_hook_record()
    ptrs = [c.region_alloc(s) for s in _alloc_sizes(0)]
    c.end_hook_record()
    events = c.hook_events_json()
    # 2) registry: a 1 MB image
    img = os.path.join(workdir, "mock.cubin")
    with open(img, "wb") as f:
        f.write(_image_bytes(0))
    _, h = c.load_image_file(img)
    # 3) graphs: build live graphs through the driver, analyze them back, save
    record = {"ptrs": ptrs, "image_hash": h, "offset": c.get_current_alloc_offset(), "graphs": []}
    for gi in range(N_GRAPHS):
        desc = c.graph_from_json_text(_graph_json(gi, h, ptrs))
        c.recompute_topology_key(desc)
        live = c.build_live_graph(desc)
        analyzed = c.analyze_graph(live)
        c.destroy_graph(live)
        if gi == 0:
            analyzed.allocator_events_json = events
        path = os.path.join(archive, f"graph_{gi}.json")
        analyzed.save(path)
        record["graphs"].append({"path": path, "json": analyzed.to_json(), "key": analyzed.topology_key})
    fb.pack_fatbins_to_folder(archive)
    from foundry_b200.graphs import save_graph_manifest

    manifest = save_graph_manifest(archive)
    assert len(manifest["topology_groups"]) == N_GROUPS, manifest
    with open(os.path.join(workdir, "record.json"), "w") as f:
        json.dump(record, f)
    print("SAVE OK", len(ptrs), hex(h))


def scenario_load(workdir: str) -> None:
    fb, c = _core()
    with open(os.path.join(workdir, "record.json")) as f:
        record = json.load(f)
    archive = os.path.join(workdir, "archive")
    fb.load_cuda_modules_and_libraries(archive)
    c.set_allocation_region(BASE, REGION)
    paths = [g["path"] for g in record["graphs"]]
    # binary files must decode to exactly what SAVE analyzed
    for g in record["graphs"]:
        d = c.read_binary_graph(g["path"].replace(".json", ".cugraph"))
        assert d.to_json() == g["json"], f"binary round trip differs for {g['path']}"
    pending = c.start_graph_builds(paths, 4)
    pending.wait()
    assert pending.num_groups == N_GROUPS, pending.num_groups
    graphs = [pending.finish_one(i) for i in range(len(paths))]
    # allocator events of graph 0 replayed -> same 200 addresses, same cursor
    assert c.get_current_alloc_offset() == record["offset"], (c.get_current_alloc_offset(), record["offset"])
    ev = json.loads(graphs[0].desc.allocator_events_json)
    assert [e["ptr"] for e in ev["events"]] == record["ptrs"]
    templates = sum(1 for g in graphs if g.is_template)
    assert templates == N_GROUPS
    for g, rec in zip(graphs, record["graphs"]):
        assert g.desc.topology_key == rec["key"]
        g.launch(0)  # mock: runs nodes in order, patches on-demand members
    # every member's launch state equals its own saved parameters
    for g, rec in zip(graphs, record["graphs"]):
        g.launch(0)
    # a background thread gives every member its own executable while the
    # main thread keeps launching them (template patching or own exec)
    import threading

    errors = []

    def materialize_all():
        try:
            for g in graphs:
                g.materialize()
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append(e)

    t = threading.Thread(target=materialize_all)
    t.start()
    for _ in range(10):
        for g in graphs:
            g.launch(0)
    t.join()
    assert not errors, errors
    assert all(g.materialized for g in graphs)
    for g in graphs:
        g.launch(0)
    # the image came back byte-identical (same CRC-64 hash re-registered)
    _, h = c.load_image_file(os.path.join(workdir, "mock.cubin"))
    assert h == record["image_hash"]
    assert c.registry_count() >= 1
    print("LOAD OK", len(graphs), templates, pending.phase1_ms, pending.phase2_ms)


def _cluster_graph_json(img_hash: int, ptrs: list[int], cluster: int | None, seed: int) -> str:
    """Four kernels; node 2 launches with a (cluster, 1, 1) cluster when
    ``cluster`` is set (the shape of the two-SM GEMM's launch)."""
    rnd = random.Random(seed)
    nodes = []
    for n in range(4):
        params, off = [], 0
        for i, sz in enumerate(PARAM_SIZES):
            val = struct.pack("<Q", ptrs[rnd.randrange(len(ptrs))]) if (sz == 8 and i < 3) else \
                bytes(rnd.getrandbits(8) for _ in range(sz))
            params.append({"index": i, "offset": off, "size": sz, "value_hex": val.hex()})
            off += sz
        node = {"id": n, "type": "KernelNode", "params": {
            "blockDimX": 192, "blockDimY": 1, "blockDimZ": 1, "gridDimX": 2 * (1 + rnd.randrange(74)),
            "gridDimY": 1, "gridDimZ": 1, "sharedMemBytes": 0, "kernelParams": params,
            "function_name": f"fbmock_k{n}", "kernel_source_binary_hash": f"{img_hash:016x}"}}
        if n == 2 and cluster:
            node["params"]["kernel_node_attrs"] = {"attrQueryAvailable": 1, "clusterDimX": cluster,
                                                   "clusterDimY": 1, "clusterDimZ": 1}
        nodes.append(node)
    deps = [{"from": i, "to": i + 1} for i in range(3)]
    return json.dumps({"nodes": nodes, "dependencies": deps, "topology_key": "", "generators": []})


def scenario_cluster(workdir: str) -> None:
    """Cluster launch dimensions survive analysis, JSON and .cugraph, restore
    onto the rebuilt node, and split topology groups: graphs 0 and 2 (node 2
    in 2-CTA clusters) share a template, graph 1 (no cluster) does not."""
    fb, c = _core()
    phase = sys.argv[3]
    archive = os.path.join(workdir, "cluster_archive")
    img = os.path.join(workdir, "mock.cubin")
    if phase == "save":
        os.makedirs(archive, exist_ok=True)
        c.set_allocation_region(BASE, REGION)
        ptrs = [c.region_alloc(1 << 20) for _ in range(8)]
        with open(img, "wb") as f:
            f.write(_image_bytes(0))
        _, h = c.load_image_file(img)
        keys = []
        for gi, cl in enumerate((2, None, 2)):
            desc = c.graph_from_json_text(_cluster_graph_json(h, ptrs, cl, 50 + gi))
            c.recompute_topology_key(desc)
            live = c.build_live_graph(desc)
            analyzed = c.analyze_graph(live)
            c.destroy_graph(live)
            node2 = json.loads(analyzed.to_json())["nodes"][2]["params"]
            if cl:
                attrs = node2.get("kernel_node_attrs") or json.loads(analyzed.to_json()).get("common_kernel_node_attrs")
                assert attrs and attrs["clusterDimX"] == 2, node2
            keys.append(analyzed.topology_key)
            analyzed.save(os.path.join(archive, f"graph_{gi}.json"))
        assert ":C2_1_1" in keys[0] and ":C2_1_1" not in keys[1] and keys[0] == keys[2], keys
        fb.pack_fatbins_to_folder(archive)
        from foundry_b200.graphs import save_graph_manifest

        m = save_graph_manifest(archive)
        assert len(m["topology_groups"]) == 2, m
        with open(os.path.join(workdir, "cluster_keys.json"), "w") as f:
            json.dump(keys, f)
        print("CLUSTER SAVE OK")
        return
    keys = json.load(open(os.path.join(workdir, "cluster_keys.json")))
    fb.load_cuda_modules_and_libraries(archive)
    c.set_allocation_region(BASE, REGION)
    paths = [os.path.join(archive, f"graph_{i}.json") for i in range(3)]
    for p, k in zip(paths, keys):
        d = c.read_binary_graph(p.replace(".json", ".cugraph"))
        assert d.topology_key == k
    pending = c.start_graph_builds(paths, 2)
    pending.wait()
    assert pending.num_groups == 2, pending.num_groups
    graphs = [pending.finish_one(i) for i in range(3)]
    for g, k in zip(graphs, keys):
        assert g.desc.topology_key == k
        g.launch(0)
    print("CLUSTER LOAD OK")


def _mixed_graph_json(img_hash: int, ptrs: list[int]) -> str:
    """kernel -> memcpy (device to device) -> event record -> empty -> event
    wait -> memset -> kernel: every node type the graph store handles."""
    def kernel(i, seed):
        rnd = random.Random(seed)
        params, off = [], 0
        for j, sz in enumerate(PARAM_SIZES):
            val = struct.pack("<Q", ptrs[j % len(ptrs)]) if (sz == 8 and j < 3) else \
                bytes(rnd.getrandbits(8) for _ in range(sz))
            params.append({"index": j, "offset": off, "size": sz, "value_hex": val.hex()})
            off += sz
        return {"id": i, "type": "KernelNode", "params": {
            "blockDimX": 64, "blockDimY": 1, "blockDimZ": 1, "gridDimX": 8, "gridDimY": 1, "gridDimZ": 1,
            "sharedMemBytes": 0, "kernelParams": params, "function_name": "fbmock_k1",
            "kernel_source_binary_hash": f"{img_hash:016x}"}}
    memcpy = {k: 0 for k in ("Depth", "Height", "WidthInBytes", "dstDevice", "dstHeight", "dstLOD", "dstPitch",
                             "dstXInBytes", "dstY", "dstZ", "srcDevice", "srcHeight", "srcLOD", "srcPitch",
                             "srcXInBytes", "srcY", "srcZ")}
    memcpy.update({"Depth": 1, "Height": 1, "WidthInBytes": 4096, "dstDevice": ptrs[1], "srcDevice": ptrs[0],
                   "dstMemoryType": 2, "srcMemoryType": 2})
    nodes = [kernel(0, 7), {"id": 1, "type": "MemcpyNode", "params": memcpy},
             {"id": 2, "type": "EventRecordNode", "params": {"event_id": 0}},
             {"id": 3, "type": "EmptyNode", "params": {}},
             {"id": 4, "type": "EventWaitNode", "params": {"event_id": 0}},
             {"id": 5, "type": "MemsetNode", "params": {"dst": ptrs[2], "elementSize": 4, "height": 1, "pitch": 0,
                                                        "value": 0xABCD, "width": 256}},
             kernel(6, 8)]
    deps = [{"from": i, "to": i + 1} for i in range(6)]
    return json.dumps({"nodes": nodes, "dependencies": deps, "topology_key": "", "generators": [],
                       "num_events": 1})


def scenario_mixed(workdir: str) -> None:
    """Memcpy, event record / wait, empty and memset nodes next to kernels:
    analysis reads them back, JSON and .cugraph round-trip them, and a fresh
    process restores and launches the graph."""
    fb, c = _core()
    phase = sys.argv[3]
    archive = os.path.join(workdir, "mixed_archive")
    img = os.path.join(workdir, "mock.cubin")
    if phase == "save":
        os.makedirs(archive, exist_ok=True)
        c.set_allocation_region(BASE, REGION)
        ptrs = [c.region_alloc(1 << 20) for _ in range(3)]
        with open(img, "wb") as f:
            f.write(_image_bytes(0))
        _, h = c.load_image_file(img)
        desc = c.graph_from_json_text(_mixed_graph_json(h, ptrs))
        c.recompute_topology_key(desc)
        live = c.build_live_graph(desc)
        analyzed = c.analyze_graph(live)
        c.destroy_graph(live)
        got = json.loads(analyzed.to_json())
        types = [n["type"] for n in got["nodes"]]
        assert types == ["KernelNode", "MemcpyNode", "EventRecordNode", "EmptyNode", "EventWaitNode", "MemsetNode",
                         "KernelNode"], types
        assert got["nodes"][1]["params"]["WidthInBytes"] == 4096 and got["nodes"][1]["params"]["srcDevice"] == ptrs[0]
        assert got["nodes"][5]["params"]["value"] == 0xABCD and got["num_events"] == 1
        assert got["nodes"][2]["params"]["event_id"] == got["nodes"][4]["params"]["event_id"]
        path = os.path.join(archive, "graph_0.json")
        analyzed.save(path)
        fb.pack_fatbins_to_folder(archive)
        with open(os.path.join(workdir, "mixed.json"), "w") as f:
            json.dump({"json": analyzed.to_json(), "key": analyzed.topology_key}, f)
        print("MIXED SAVE OK")
        return
    rec = json.load(open(os.path.join(workdir, "mixed.json")))
    fb.load_cuda_modules_and_libraries(archive)
    c.set_allocation_region(BASE, REGION)
    for _ in range(3):
        c.region_alloc(1 << 20)
    path = os.path.join(archive, "graph_0.json")
    assert c.read_binary_graph(path.replace(".json", ".cugraph")).to_json() == rec["json"]
    pending = c.start_graph_builds([path], 1)
    g = pending.finish_one(0)
    assert g.desc.topology_key == rec["key"]
    g.launch(0)
    g.materialize()
    g.launch(0)
    # without the binary file the JSON is read instead, to the same description
    os.remove(path.replace(".json", ".cugraph"))
    assert c.read_graph_file(path).to_json() == rec["json"]
    g2 = c.start_graph_builds([path], 1).finish_one(0)
    assert g2.desc.topology_key == rec["key"]
    g2.launch(0)
    print("MIXED LOAD OK")


def scenario_pdl(workdir: str) -> None:
    """Programmatic dependent launch edges (edge data: ports and type) are read
    with the v2 edge query, kept in JSON and .cugraph, enter the topology key
    and are re-created on restore; a graph of such edges is not grouped with
    the same graph of plain edges."""
    fb, c = _core()
    archive = os.path.join(workdir, "pdl_archive")
    os.makedirs(archive, exist_ok=True)
    c.set_allocation_region(BASE, REGION)
    ptrs = [c.region_alloc(1 << 20) for _ in range(3)]
    img = os.path.join(workdir, "mock.cubin")
    with open(img, "wb") as f:
        f.write(_image_bytes(0))
    _, h = c.load_image_file(img)
    base = json.loads(_mixed_graph_json(h, ptrs))
    nodes = [base["nodes"][0], dict(base["nodes"][6], id=1), dict(base["nodes"][0], id=2)]
    # kernel 0 -> kernel 1: programmatic (from_port 1 = programmatic port, type 1 = programmatic);
    # kernel 1 -> kernel 2: plain
    pdl = {"nodes": nodes, "dependencies": [{"from": 0, "to": 1, "from_port": 1, "to_port": 0, "type": 1},
                                            {"from": 1, "to": 2}], "topology_key": "", "generators": [],
           "num_events": 0}
    plain = dict(pdl, dependencies=[{"from": 0, "to": 1}, {"from": 1, "to": 2}])
    keys = {}
    for name, doc in (("pdl", pdl), ("plain", plain)):
        desc = c.graph_from_json_text(json.dumps(doc))
        c.recompute_topology_key(desc)
        live = c.build_live_graph(desc)
        analyzed = c.analyze_graph(live)
        c.destroy_graph(live)
        got = json.loads(analyzed.to_json())
        deps = sorted((d["from"], d["to"], d.get("from_port", 0), d.get("type", 0)) for d in got["dependencies"])
        want = [(0, 1, 1, 1), (1, 2, 0, 0)] if name == "pdl" else [(0, 1, 0, 0), (1, 2, 0, 0)]
        assert deps == want, (name, deps)
        keys[name] = analyzed.topology_key
        path = os.path.join(archive, f"graph_{len(keys) - 1}.json")
        analyzed.save(path)
        assert c.read_binary_graph(path.replace(".json", ".cugraph")).to_json() == analyzed.to_json()
    assert keys["pdl"] != keys["plain"], keys
    paths = [os.path.join(archive, "graph_0.json"), os.path.join(archive, "graph_1.json")]
    pending = c.start_graph_builds(paths, 2)
    pending.wait()
    assert pending.num_groups == 2
    for i in range(2):
        g = pending.finish_one(i)
        g.launch(0)
        g.materialize()
        g.launch(0)
    print("PDL OK")


def scenario_numeric(workdir: str) -> None:
    """A graph of axpy/fill kernels on region memory: SAVE runs it, LOAD restores
    and runs it again; results must be bit-identical."""
    fb, c = _core()
    import ctypes

    mode = sys.argv[3]
    archive = os.path.join(workdir, "num_archive")
    os.makedirs(archive, exist_ok=True)
    if mode == "load":
        fb.load_cuda_modules_and_libraries(archive)
    c.set_allocation_region(BASE, REGION)
    n = 4096
    y, x = c.region_alloc(4 * n), c.region_alloc(4 * n)
    xs = (ctypes.c_float * n).from_address(x)
    ys = (ctypes.c_float * n).from_address(y)
    for i in range(n):
        xs[i] = 0.5 * i
        ys[i] = 1.0
    img = os.path.join(workdir, "mock.cubin")
    with open(img, "wb") as f:
        f.write(_image_bytes(0))
    _, h = c.load_image_file(img)
    nodes = []
    for j in range(6):
        a = struct.pack("<f", 0.25 * (j + 1))
        nodes.append({"id": j, "type": "KernelNode", "params": {
            "blockDimX": 128, "blockDimY": 1, "blockDimZ": 1, "gridDimX": 32, "gridDimY": 1, "gridDimZ": 1,
            "sharedMemBytes": 0, "function_name": "fbmock_axpy_f32", "kernel_source_binary_hash": f"{h:016x}",
            "kernelParams": [
                {"value_hex": struct.pack("<Q", y).hex()}, {"value_hex": struct.pack("<Q", x).hex()},
                {"value_hex": a.hex()}, {"value_hex": struct.pack("<I", n).hex()}]}})
    text = json.dumps({"nodes": nodes, "dependencies": [{"from": i, "to": i + 1} for i in range(5)],
                       "topology_key": "", "generators": []})
    path = os.path.join(archive, "graph_0.json")
    if mode == "save":
        desc = c.graph_from_json_text(text)
        c.recompute_topology_key(desc)
        live = c.build_live_graph(desc)
        d2 = c.analyze_graph(live)
        c.destroy_graph(live)
        d2.save(path)
        fb.pack_fatbins_to_folder(archive)
    g = c.load_graph(path)
    g.launch(0)
    g.launch(0)
    vals = [ys[i] for i in range(0, n, 97)]
    with open(os.path.join(workdir, f"num_{mode}.json"), "w") as f:
        json.dump(vals, f)
    print("NUMERIC", mode, vals[:3])


def scenario_faults(workdir: str) -> None:
    """Host-side fault injection: corrupt archive, wrong hash, missing entry point,
    cursor drift. Every failure must surface as a Python exception (status), never
    an abort."""
    fb, c = _core()
    import shutil

    archive = os.path.join(workdir, "archive")
    bad = os.path.join(workdir, "bad_archive")
    shutil.copytree(archive, bad)
    # (a) corrupted image bytes -> CRC mismatch
    p = os.path.join(bad, "fatbin_image_packed.img")
    data = bytearray(open(p, "rb").read())
    data[100] ^= 0xFF
    open(p, "wb").write(bytes(data))
    try:
        fb.load_cuda_modules_and_libraries(bad)
        raise AssertionError("corrupt image was accepted")
    except RuntimeError as e:
        assert "CRC" in str(e), e
    # (b) truncated image file
    open(p, "wb").write(bytes(data[:50]))
    try:
        fb.load_cuda_modules_and_libraries(bad)
        raise AssertionError("truncated pack was accepted")
    except RuntimeError as e:
        assert "truncated" in str(e), e
    # (c) truncated .cugraph
    g0 = os.path.join(archive, "graph_1.cugraph")
    tb = os.path.join(workdir, "trunc.cugraph")
    open(tb, "wb").write(open(g0, "rb").read()[:200])
    try:
        c.read_binary_graph(tb)
        raise AssertionError("truncated graph accepted")
    except RuntimeError as e:
        assert "corrupt" in str(e), e
    # (d) graph whose image was never loaded (wrong hash) -> not found
    fb.load_cuda_modules_and_libraries(archive)
    c.set_allocation_region(BASE, REGION)
    with open(os.path.join(archive, "graph_1.json")) as f:
        j = json.load(f)
    j["nodes"][1]["params"]["kernel_source_binary_hash"] = "deadbeefdeadbeef"
    wrong = os.path.join(workdir, "wrong_hash.json")
    json.dump(j, open(wrong, "w"))
    try:
        c.load_graph(wrong)
        raise AssertionError("unknown image accepted")
    except RuntimeError as e:
        assert "not loaded" in str(e), e
    # (e) missing entry point
    with open(os.path.join(archive, "graph_1.json")) as f:
        j = json.load(f)
    j["nodes"][1]["params"]["function_name"] = "fbmock_missing"
    missing = os.path.join(workdir, "missing_entry.json")
    json.dump(j, open(missing, "w"))
    try:
        c.load_graph(missing)
        raise AssertionError("missing entry point accepted")
    except RuntimeError as e:
        assert "not found" in str(e), e
    # (f) cursor drift: allocate first, then replay events that started earlier
    c.region_alloc(512 << 20)
    with open(os.path.join(archive, "graph_0.json")) as f:
        ev = json.dumps(json.load(f)["allocator_events"])
    try:
        c.replay_hook_events_json(ev)
        raise AssertionError("cursor drift not detected")
    except RuntimeError as e:
        assert "drift" in str(e), e
    # (g) set_current_alloc_offset backwards is rejected
    try:
        c.set_current_alloc_offset(0)
        raise AssertionError("backwards offset accepted")
    except RuntimeError as e:
        assert "forward" in str(e), e
    # (h) a stale manifest that groups two graphs with the same node count but
    # different topology keys (groups 0 and 1 put their memset at different
    # positions) must be refused, not patched onto the wrong template
    stale = os.path.join(workdir, "stale_manifest")
    shutil.copytree(archive, stale)
    k0 = c.read_binary_graph(os.path.join(stale, "graph_0.cugraph")).topology_key
    k1 = c.read_binary_graph(os.path.join(stale, "graph_1.cugraph")).topology_key
    assert k0 != k1
    with open(os.path.join(stale, "graph_manifest.json"), "w") as f:
        json.dump({"topology_groups": [{"topology_key": k0, "template": "graph_0.json",
                                        "members": ["graph_0.json", "graph_1.json"]}]}, f)
    pending = c.start_graph_builds([os.path.join(stale, "graph_0.json"), os.path.join(stale, "graph_1.json")], 2)
    try:
        pending.wait()
        raise AssertionError("stale manifest accepted")
    except RuntimeError as e:
        assert "another topology" in str(e), e
    print("FAULTS OK")


def scenario_rng(workdir: str) -> None:
    """Generator records with seed/offset word addresses survive JSON and
    .cugraph, and relocation rewrites exactly the kernel-parameter words that
    hold those addresses (in the template and in a restore)."""
    fb, c = _core()
    archive = os.path.join(workdir, "archive")
    with open(os.path.join(archive, "graph_1.json")) as f:
        j = json.load(f)
    # graph_1's first kernel node: its first parameter is a region pointer
    k = next(n for n in j["nodes"] if n["type"] == "KernelNode")
    seed_ptr = struct.unpack("<Q", bytes.fromhex(k["params"]["kernelParams"][0]["value_hex"]))[0]
    offset_ptr = struct.unpack("<Q", bytes.fromhex(k["params"]["kernelParams"][1]["value_hex"]))[0]
    assert seed_ptr != offset_ptr
    hits = sum(1 for n in j["nodes"] if n["type"] == "KernelNode" for prm in n["params"]["kernelParams"]
               if prm["size"] == 8 and struct.unpack("<Q", bytes.fromhex(prm["value_hex"]))[0] in (seed_ptr, offset_ptr))
    d = c.graph_from_json_text(json.dumps(j))
    d.generators = [{"id": 0, "seed": 42, "wholegraph_increment": 8, "seed_ptr": seed_ptr, "offset_ptr": offset_ptr}]
    out = os.path.join(workdir, "rng", "graph_0.json")
    os.makedirs(os.path.dirname(out), exist_ok=True)
    d.save(out)
    for rd in (c.read_binary_graph(out.replace(".json", ".cugraph")),
               c.graph_from_json_text(open(out).read())):
        assert rd.generators == [{"id": 0, "seed": 42, "wholegraph_increment": 8, "seed_ptr": seed_ptr,
                                  "offset_ptr": offset_ptr}], rd.generators
    slot = 0x7F0000001000
    rd = c.read_binary_graph(out.replace(".json", ".cugraph"))
    n = rd.relocate_generator_words(slot)
    assert n == hits and n >= 2, (n, hits)
    assert rd.generators[0]["seed_ptr"] == slot and rd.generators[0]["offset_ptr"] == slot + 8
    rel = json.loads(rd.to_json())
    for a, b in zip(j["nodes"], rel["nodes"]):
        if a["type"] != "KernelNode":
            continue
        for pa, pb in zip(a["params"]["kernelParams"], b["params"]["kernelParams"]):
            va, vb = bytes.fromhex(pa["value_hex"]), bytes.fromhex(pb["value_hex"])
            if pa["size"] == 8 and struct.unpack("<Q", va)[0] == seed_ptr:
                assert struct.unpack("<Q", vb)[0] == slot
            elif pa["size"] == 8 and struct.unpack("<Q", va)[0] == offset_ptr:
                assert struct.unpack("<Q", vb)[0] == slot + 8
            else:
                assert va == vb
    # a graph without generator addresses keeps the 24-byte v1 records
    d.generators = [{"id": 0, "seed": 1, "wholegraph_increment": 4}]
    d.save(out)
    assert c.read_binary_graph(out.replace(".json", ".cugraph")).generators[0]["seed_ptr"] == 0
    print("RNG OK", n)


if __name__ == "__main__":
    name, workdir = sys.argv[1], sys.argv[2]
    {"save": scenario_save, "load": scenario_load, "numeric": scenario_numeric, "faults": scenario_faults,
     "cluster": scenario_cluster, "mixed": scenario_mixed, "rng": scenario_rng, "pdl": scenario_pdl}[name](workdir)
