"""CPU tests of the offline-format layer of libdvs_b200.so (no GPU needed)."""
import filecmp
import json
import os
import struct

import numpy as np
import pytest

from conftest import uniform_int_data, write_oracle_index


@pytest.fixture(scope="module")
def small_index(oracle):
    X = uniform_int_data(700, 20, 3)
    return oracle.build_index(X, R=12, L=24)


@pytest.mark.parametrize("M", [1, 2, 5])
def test_reader_matches_oracle_writer(oracle, dvs, small_index, tmp_path, M):
    idx = small_index
    pre = write_oracle_index(oracle, idx, str(tmp_path / "a" / "idx"), M)
    info, adj, rec, vec, ids, P, c = dvs.load_host_index(pre)
    assert (info.num_vectors, info.dim, info.R, info.rabitq_bits, info.num_memory_nodes) == (700, 20, 12, 4, M)
    assert info.rabitq_size == oracle.rabitq_size(20, 4)
    assert info.medoid == idx.medoid and info.t_const == idx.t_const
    np.testing.assert_array_equal(adj, idx.adj)
    np.testing.assert_array_equal(rec, idx.records)
    np.testing.assert_array_equal(vec, idx.X)
    np.testing.assert_array_equal(ids, np.arange(700))
    np.testing.assert_array_equal(P, idx.P)
    np.testing.assert_array_equal(c, idx.c_rot)


@pytest.mark.parametrize("M", [1, 3])
def test_writer_is_byte_identical_to_oracle_writer(oracle, dvs, small_index, tmp_path, M):
    idx = small_index
    a = write_oracle_index(oracle, idx, str(tmp_path / "a" / "idx"), M)
    b = str(tmp_path / "b" / "idx")
    dvs.write_index(b, idx.X, idx.adj, idx.records, idx.P, idx.c_rot, idx.medoid, idx.t_const, 4, num_memory_nodes=M)
    for s in range(M):
        assert filecmp.cmp(f"{a}_node{s + 1}_of{M}.dat", f"{b}_node{s + 1}_of{M}.dat", shallow=False)
    assert filecmp.cmp(a + ".rotation.bin", b + ".rotation.bin", shallow=False)
    ma, mb = json.load(open(a + ".meta.json")), json.load(open(b + ".meta.json"))
    for key in ("R", "dim", "rabitq_bits", "num_memory_nodes", "rabitq_size", "node_size", "medoid", "num_vectors"):
        assert ma[key] == mb[key]


def test_node_record_layout(oracle, small_index, tmp_path):
    """VamanaNode layout (src/vamana/vamana_node.hh:10-69) and placement
    (node i in shard i mod M at 16 + (i div M) * align8(node_size))."""
    idx, M = small_index, 3
    pre = write_oracle_index(oracle, idx, str(tmp_path / "idx"), M)
    node_size = 16 + 4 * 20 + oracle.rabitq_size(20, 4) + 8 * 12
    aligned = (node_size + 7) & ~7
    raw = open(f"{pre}_node2_of3.dat", "rb").read()
    i = 7  # shard 1, slot 2
    off = 16 + (i // M) * aligned
    assert struct.unpack_from("<I", raw, off + 8)[0] == i
    ec = raw[off + 12]
    assert ec == (idx.adj[i] != oracle.EMPTY).sum()
    vec = np.frombuffer(raw, np.float32, 20, off + 16)
    np.testing.assert_array_equal(vec, idx.X[i])
    nb = struct.unpack_from(f"<{ec}Q", raw, off + 16 + 80 + oracle.rabitq_size(20, 4))
    for j, p in enumerate(nb):
        t = int(idx.adj[i][j])
        assert p >> 48 == t % M and (p & ((1 << 48) - 1)) == 16 + (t // M) * aligned
    header0 = open(f"{pre}_node1_of3.dat", "rb").read(16)
    free_ptr, medoid_ptr = struct.unpack("<QQ", header0)
    assert medoid_ptr >> 48 == idx.medoid % M


def _expect(dvs, pre, name):
    with pytest.raises(dvs.DvsError) as e:
        dvs.load_host_index(pre)
    assert e.value.name == name, str(e.value)


def _corrupt_index(oracle, idx, tmp_path, name, M=1):
    return write_oracle_index(oracle, idx, str(tmp_path / name / "idx"), M)


def test_missing_files(oracle, dvs, small_index, tmp_path):
    _expect(dvs, str(tmp_path / "nothing" / "idx"), "DVS_ERR_IO")
    pre = _corrupt_index(oracle, small_index, tmp_path, "norot")
    os.remove(pre + ".rotation.bin")
    _expect(dvs, pre, "DVS_ERR_IO")
    pre = _corrupt_index(oracle, small_index, tmp_path, "noshard", M=2)
    os.remove(pre + "_node2_of2.dat")
    _expect(dvs, pre, "DVS_ERR_IO")


def _edit_meta(pre, **kv):
    m = json.load(open(pre + ".meta.json"))
    for k, v in kv.items():
        if v is None:
            m.pop(k)
        else:
            m[k] = v
    json.dump(m, open(pre + ".meta.json", "w"))


@pytest.mark.parametrize("edit,name", [
    ({"dim": None}, "DVS_ERR_FORMAT"),
    ({"rabitq_bits": 3}, "DVS_ERR_BITS"),
    ({"rabitq_size": 99}, "DVS_ERR_FORMAT"),
    ({"num_memory_nodes": 0}, "DVS_ERR_FORMAT"),
    ({"distance": "cosine"}, "DVS_ERR_FORMAT"),
    ({"R": 300}, "DVS_ERR_FORMAT"),
    ({"dim": 21}, "DVS_ERR_DIM"),
])
def test_bad_metadata(oracle, dvs, small_index, tmp_path, edit, name):
    pre = _corrupt_index(oracle, small_index, tmp_path, "meta")
    _edit_meta(pre, **edit)
    _expect(dvs, pre, name)


def test_not_json(oracle, dvs, small_index, tmp_path):
    pre = _corrupt_index(oracle, small_index, tmp_path, "nj")
    open(pre + ".meta.json", "w").write("{dim: 3")
    _expect(dvs, pre, "DVS_ERR_FORMAT")


def test_truncated_rotation(oracle, dvs, small_index, tmp_path):
    pre = _corrupt_index(oracle, small_index, tmp_path, "rot")
    raw = open(pre + ".rotation.bin", "rb").read()
    open(pre + ".rotation.bin", "wb").write(raw[:-9])
    _expect(dvs, pre, "DVS_ERR_FORMAT")
    open(pre + ".rotation.bin", "wb").write(struct.pack("<I", 19) + raw[4:])
    _expect(dvs, pre, "DVS_ERR_DIM")


def _patch_shard(path, off, data):
    raw = bytearray(open(path, "rb").read())
    raw[off:off + len(data)] = data
    open(path, "wb").write(bytes(raw))


def test_corrupt_shards(oracle, dvs, small_index, tmp_path):
    idx = small_index
    node_size = 16 + 4 * 20 + oracle.rabitq_size(20, 4) + 8 * 12
    aligned = (node_size + 7) & ~7
    nb_off = 16 + 80 + oracle.rabitq_size(20, 4)
    # free pointer not on a node boundary
    pre = _corrupt_index(oracle, idx, tmp_path, "fp")
    _patch_shard(pre + "_node1_of1.dat", 0, struct.pack("<Q", 17))
    _expect(dvs, pre, "DVS_ERR_FORMAT")
    # neighbour pointer outside the shards
    pre = _corrupt_index(oracle, idx, tmp_path, "nb")
    _patch_shard(pre + "_node1_of1.dat", 16 + 5 * aligned + nb_off, struct.pack("<Q", (7 << 48) | 16))
    _expect(dvs, pre, "DVS_ERR_FORMAT")
    # neighbour pointer inside a node
    pre = _corrupt_index(oracle, idx, tmp_path, "mid")
    _patch_shard(pre + "_node1_of1.dat", 16 + 5 * aligned + nb_off, struct.pack("<Q", 16 + 3))
    _expect(dvs, pre, "DVS_ERR_FORMAT")
    # edge count above R
    pre = _corrupt_index(oracle, idx, tmp_path, "ec")
    _patch_shard(pre + "_node1_of1.dat", 16 + 2 * aligned + 12, bytes([13]))
    _expect(dvs, pre, "DVS_ERR_FORMAT")
    # null medoid pointer
    pre = _corrupt_index(oracle, idx, tmp_path, "med")
    _patch_shard(pre + "_node1_of1.dat", 8, struct.pack("<Q", 0))
    _expect(dvs, pre, "DVS_ERR_FORMAT")
    # non-finite vector component
    pre = _corrupt_index(oracle, idx, tmp_path, "nan")
    _patch_shard(pre + "_node1_of1.dat", 16 + 4 * aligned + 16, struct.pack("<f", float("nan")))
    _expect(dvs, pre, "DVS_ERR_FORMAT")


def test_null_neighbour_slots_are_skipped(oracle, dvs, small_index, tmp_path):
    """A null RemotePtr inside edge_count is skipped (src/vamana/vamana.hh:177)."""
    idx = small_index
    node_size = 16 + 4 * 20 + oracle.rabitq_size(20, 4) + 8 * 12
    aligned = (node_size + 7) & ~7
    nb_off = 16 + 80 + oracle.rabitq_size(20, 4)
    pre = _corrupt_index(oracle, idx, tmp_path, "null")
    _patch_shard(pre + "_node1_of1.dat", 16 + 9 * aligned + nb_off, struct.pack("<Q", 0))
    _, adj, *_ = dvs.load_host_index(pre)
    row = idx.adj[9][idx.adj[9] != oracle.EMPTY]
    got = adj[9][adj[9] != oracle.EMPTY]
    np.testing.assert_array_equal(got, row[1:])
