"""Helpers the tests share for a conversation's state in the oracle's arrays (no test of its own)."""
import numpy as np


def compact_kv(ora, st):
    """The oracle's KV arrays ([layer][K|V][ctx][row]) cut to the positions held, as the state bridge takes them."""
    c = ora.cfg
    A = max(1, ora.n_attn)
    row = c.n_kv_heads * c.head_dim
    if ora.n_attn == 0:
        return np.zeros((1, 2, st.pos, row), np.int8), np.zeros((1, 2, st.pos, c.n_kv_heads), np.float32)
    kv = st.kv.reshape(A, 2, st.ctx, row)[:, :, :st.pos].copy()
    kvs = st.kvs.reshape(A, 2, st.ctx, c.n_kv_heads)[:, :, :st.pos].copy()
    return kv, kvs


def random_state(ora, st, positions, rng):
    """positions of random int8 KV rows (scales U(0.005, 0.02)), random conv and recurrent states."""
    c = ora.cfg
    A = max(1, ora.n_attn)
    row = c.n_kv_heads * c.head_dim
    kv = st.kv.reshape(A, 2, st.ctx, row)
    kvs = st.kvs.reshape(A, 2, st.ctx, c.n_kv_heads)
    if ora.n_attn:
        kv[:, :, :positions] = rng.integers(-127, 128, kv[:, :, :positions].shape, dtype=np.int8)
        kvs[:, :, :positions] = rng.uniform(0.005, 0.02, kvs[:, :, :positions].shape).astype(np.float32)
    if ora.n_gdn:
        st.conv[:] = (rng.standard_normal(st.conv.shape) * 0.3).astype(np.float32)
        st.gdn[:] = (rng.standard_normal(st.gdn.shape) * 0.02).astype(np.float32)
    st.pos = positions
