"""V3-OT function-table lookups, the server's side on the GPU, against the oracle:

* StandardOtTables (crates/v2/sharing/src/secure_nonlinear_ot.rs:44-72,554-575): the device
  tables bit-exact with the oracle's restatement of OtFunctionTable::new (f32 arithmetic and libm
  as the Rust code), and the reference's own unit-test facts (index of 0, -8, 8; SiLU(0) ~ 0);
* IknpOtExtension::process_query (crates/ot/src/iknp.rs:495-572) on the GPU, byte-exact with the
  oracle's Python restatement over hashlib SHA-256 and AES-128, for batches of 1 to 4000 entries;
  the client's decode of the response recovers exactly the table rows it asked for;
* errors: InvalidIndex for the first out-of-range entry, InvalidMessageFormat for a bad length.
"""
import os

import numpy as np
import pytest

gpu = pytest.mark.gpu


def test_oracle_tables_reference_facts(orc):
    """secure_nonlinear_ot.rs test_ot_function_table, restated (CPU)."""
    t = orc.ot_standard_tables(1024)
    assert orc.ot_input_to_index(0.0, 0, 1024) == 512
    assert orc.ot_input_to_index(-8.0, 0, 1024) == 0
    assert orc.ot_input_to_index(8.0, 0, 1024) == 1023
    assert abs(float(t[0][512])) < 0.01
    # out-of-range inputs clamp; NaN maps to index 0 (Rust's saturating cast)
    assert orc.ot_input_to_index(100.0, 1, 4096) == 4095 and orc.ot_input_to_index(float("nan"), 2, 4096) == 0


def test_oracle_ot_round_trip(orc):
    """generate_query -> process_query -> decode_response returns the selected rows (CPU)."""
    rng = np.random.default_rng(0)
    t = orc.ot_standard_tables(4096)[3].tobytes()
    com, seed = os.urandom(32), os.urandom(32)
    idx = rng.integers(0, 4096, 50)
    rks = [os.urandom(16) for _ in idx]
    q = orc.ot_generate_query(com, 7, idx, seed, rks)
    got = np.frombuffer(orc.ot_decode_response(orc.ot_process_query(com, 7, q, t, 4), 7, rks, 4), np.float32)
    assert np.array_equal(got, np.frombuffer(t, np.float32)[idx])


@gpu
def test_device_tables_bit_exact(ctx, orc):
    from shardlm_b200.sharing import StandardOtTables

    for size in (1024, 4096):
        dev = StandardOtTables(ctx, size).values.cpu().numpy()
        assert np.array_equal(dev.view(np.uint32), orc.ot_standard_tables(size).view(np.uint32))


@gpu
@pytest.mark.parametrize("m,table", [(1, "silu"), (19, "rsqrt"), (777, "exp"), (4000, "reciprocal")])
def test_process_query_matches_oracle(ctx, orc, m, table):
    from shardlm_b200.sharing import OtFunctionServer, StandardOtTables

    rng = np.random.default_rng(m)
    tabs = StandardOtTables(ctx, 4096)
    t = tabs.table(table)
    t_bytes = t.cpu().numpy().tobytes()
    com = bytes(rng.integers(0, 256, 32, dtype=np.uint8))
    srv = OtFunctionServer(ctx, com)
    for _ in range(2):  # the session counter advances per query
        seed = bytes(rng.integers(0, 256, 32, dtype=np.uint8))
        idx = rng.integers(0, 4096, m)
        rks = [bytes(rng.integers(0, 256, 16, dtype=np.uint8)) for _ in range(m)]
        ctr = srv.session_ctr + 1
        q = orc.ot_generate_query(com, ctr, idx, seed, rks)
        resp = srv.process_query(q, t)
        assert resp == orc.ot_process_query(com, ctr, q, t_bytes, 4)
        vals = np.frombuffer(orc.ot_decode_response(resp, ctr, rks, 4), np.float32)
        assert np.array_equal(vals, np.frombuffer(t_bytes, np.float32)[idx])


@gpu
def test_process_query_errors(ctx, orc):
    from shardlm_b200._lib import ShdError
    from shardlm_b200.sharing import OtFunctionServer, StandardOtTables

    tabs = StandardOtTables(ctx, 1024)
    com, seed = bytes(32), bytes(range(32))
    srv = OtFunctionServer(ctx, com)
    q = orc.ot_generate_query(com, 1, [3, 1024 + 5, 2000], seed, [bytes(16)] * 3)  # entry 1 past the table
    with pytest.raises(ShdError, match="InvalidIndex at entry 1"):
        srv.process_query(q, tabs.table("silu"))
    with pytest.raises(ShdError, match="InvalidMessageFormat"):
        srv.process_query(q[:-1], tabs.table("silu"))
