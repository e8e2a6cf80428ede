"""The chip stack as sparse host tensors: every projection of every GDN + SwiGLU layer as CSR
with bf16 values, the embedding, the output head and the final norm.

This is the host-side description the table builder (``linuxformer_b200.tables``), the CPU
oracle (``oracle/``) and the stock-forward materialiser (``to_hf``) all start from. Shapes follow
the reference's chip layers (``lx/lx/hf.py:25-38, 113-118``; ``lx/lx/emit.py:216-224``):

    in_proj_qkv  (2*16*256 + 128*128 = 24576) x 2560     conv1d taps   24576 x 4
    in_proj_z    16384 x 2560                            in_proj_b/a   128 x 2560
    out_proj     2560 x 16384
    gate/up      9216 x 2560                             down          2560 x 9216

Values are bf16 bit patterns (uint16). CSR rows hold only nonzero entries, in ascending column
order; that order is the summation order every kernel and the oracle use.
"""

from __future__ import annotations

import dataclasses
import hashlib
from dataclasses import dataclass, field

import numpy as np

H = 2560          # hidden
KD, VD = 256, 128  # key / value head dims
NK, NV = 16, 128   # key / value heads
R = NV // NK       # value heads per key head
CONV = 2 * NK * KD + NV * VD  # 24576 conv channels: q | k | v
ZD = NV * VD       # 16384 value dims
INTER = 9216       # SwiGLU width
TAPS = 4


# --- bf16 helpers -------------------------------------------------------------------------------
def bf16_bits(x) -> np.ndarray:
    """float32 values -> bf16 bit patterns, round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(np.asarray(x, dtype=np.float32)).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    r = np.where(nan, (u >> 16) | 0x40, r)
    return r.astype(np.uint16)


def bf16_float(b) -> np.ndarray:
    """bf16 bit patterns -> float32."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x) -> np.ndarray:
    return bf16_float(bf16_bits(x))


# --- sparse matrices ----------------------------------------------------------------------------
@dataclass
class Sparse:
    """CSR with bf16 values: row r holds indices[indptr[r]:indptr[r+1]] (ascending columns)."""
    shape: tuple
    indptr: np.ndarray   # int64 [rows + 1]
    indices: np.ndarray  # int32 [nnz]
    data: np.ndarray     # uint16 [nnz], bf16 bits, never +-0

    @property
    def nnz(self) -> int:
        return int(self.indices.shape[0])

    @staticmethod
    def from_coo(shape, rows, cols, bits) -> "Sparse":
        rows = np.asarray(rows, np.int64)
        cols = np.asarray(cols, np.int64)
        bits = np.asarray(bits, np.uint16)
        keep = (bits & 0x7FFF) != 0
        rows, cols, bits = rows[keep], cols[keep], bits[keep]
        key = rows * shape[1] + cols
        key, first = np.unique(key, return_index=True)  # sorted, duplicates dropped
        rows, cols, bits = key // shape[1], key % shape[1], bits[first]
        indptr = np.zeros(shape[0] + 1, np.int64)
        np.cumsum(np.bincount(rows, minlength=shape[0]), out=indptr[1:])
        return Sparse(tuple(shape), indptr, cols.astype(np.int32), bits)

    @staticmethod
    def from_dense(bits2d) -> "Sparse":
        b = np.asarray(bits2d, np.uint16)
        r, c = np.nonzero(b & 0x7FFF)
        return Sparse.from_coo(b.shape, r, c, b[r, c])

    def to_dense(self) -> np.ndarray:
        out = np.zeros(self.shape, np.uint16)
        rows = np.repeat(np.arange(self.shape[0]), np.diff(self.indptr))
        out[rows, self.indices] = self.data
        return out

    def row_nnz(self) -> np.ndarray:
        return np.diff(self.indptr)

    def transpose(self) -> "Sparse":
        rows = np.repeat(np.arange(self.shape[0], dtype=np.int64), np.diff(self.indptr))
        return Sparse.from_coo((self.shape[1], self.shape[0]), self.indices, rows, self.data)

    def rows_subset(self, rows) -> "Sparse":
        rows = np.asarray(rows, np.int64)
        cnt = self.indptr[rows + 1] - self.indptr[rows]
        idx = _ranges(self.indptr[rows], cnt)
        indptr = np.zeros(len(rows) + 1, np.int64)
        np.cumsum(cnt, out=indptr[1:])
        return Sparse((len(rows), self.shape[1]), indptr, self.indices[idx], self.data[idx])


def _ranges(starts, counts) -> np.ndarray:
    """concatenation of arange(s, s + c) over the pairs (s, c)."""
    starts = np.asarray(starts, np.int64)
    counts = np.asarray(counts, np.int64)
    tot = int(counts.sum())
    if tot == 0:
        return np.zeros(0, np.int64)
    first = np.repeat(np.cumsum(counts) - counts, counts)
    return np.repeat(starts, counts) + np.arange(tot) - first


# --- the stack ----------------------------------------------------------------------------------
@dataclass
class Layer:
    """One chip layer (Qwen3_5DecoderLayer with linear_attention): GDN then SwiGLU."""
    qkv: Sparse
    conv: np.ndarray      # uint16 [CONV, 4]: conv1d.weight[:, 0, :]
    z: Sparse
    b: Sparse
    a: Sparse
    out: Sparse
    A_log: np.ndarray     # uint16 [NV]
    dt_bias: np.ndarray   # uint16 [NV]
    gnorm: np.ndarray     # uint16 [VD]: Qwen3_5RMSNormGated.weight
    ln_in: np.ndarray     # uint16 [H]: input_layernorm.weight
    ln_post: np.ndarray   # uint16 [H]: post_attention_layernorm.weight
    gate: Sparse
    up: Sparse
    down: Sparse


@dataclass
class Chip:
    name: str
    layers: list
    embed: np.ndarray     # uint16 [V_embed, H] (dense)
    head: Sparse          # [V, H]
    final_norm: np.ndarray  # uint16 [H]
    eps: float = 1e-6     # rms_norm_eps (also the gated norm's)
    offset: int = 0       # chip token t embeds row offset + t
    meta: dict = field(default_factory=dict)

    @property
    def n_layers(self) -> int:
        return len(self.layers)

    @property
    def n_vocab(self) -> int:
        return self.head.shape[0]

    def digest(self) -> str:
        """A hash of every tensor, to pin generated models against fixtures."""
        h = hashlib.sha256()
        for L in self.layers:
            for f in dataclasses.fields(L):
                v = getattr(L, f.name)
                if isinstance(v, Sparse):
                    for a in (v.indptr, v.indices, v.data):
                        h.update(np.ascontiguousarray(a).tobytes())
                else:
                    h.update(np.ascontiguousarray(v).tobytes())
        for a in (self.embed, self.head.indptr, self.head.indices, self.head.data,
                  self.final_norm):
            h.update(np.ascontiguousarray(a).tobytes())
        h.update(np.float64(self.eps).tobytes())
        return h.hexdigest()[:16]


@dataclass
class State:
    """One machine's state, in the HF cache layout (lx/lx/mega.py:506-516):
    recurrent [L][NV][KD][VD] fp32, conv [L][CONV][4] bf16 bits (oldest tap first)."""
    recurrent: np.ndarray  # float32 [L, NV, KD, VD]
    conv: np.ndarray       # uint16 [L, CONV, 4]

    def copy(self) -> "State":
        return State(self.recurrent.copy(), self.conv.copy())


# --- seeded synthetic stacks --------------------------------------------------------------------
def _sparse_random(rng, shape, density, values) -> Sparse:
    """~density * rows * cols nonzeros at uniform positions, values from values(n)."""
    n = int(round(density * shape[0] * shape[1]))
    flat = rng.integers(0, shape[0] * shape[1], size=n, dtype=np.int64)
    bits = bf16_bits(values(n))
    return Sparse.from_coo(shape, flat // shape[1], flat % shape[1], bits)


def c1(seed: int = 0, n_layers: int = 2, vocab: int = 4096, density: float = 1e-3) -> Chip:
    """Config 1: the 2-layer synthetic sparse stack. Every projection and the conv taps at
    `density` nonzeros (uniform positions), values N(0, 0.02) in bf16; embedding dense
    N(0, 0.02); output head `vocab` x 2560 at `density`. The scalar parameters are the stock
    module's own initialisation (transformers Qwen3_5GatedDeltaNet.__init__): dt_bias = 1,
    A_log = log(U(0, 16)), gated-norm weight 1, RMSNorm weights 0 (gain 1)."""
    rng = np.random.default_rng(seed)
    nrm = lambda n: rng.normal(0.0, 0.02, n)  # noqa: E731
    layers = []
    for _ in range(n_layers):
        conv = _sparse_random(rng, (CONV, TAPS), density, nrm).to_dense()
        layers.append(Layer(
            qkv=_sparse_random(rng, (CONV, H), density, nrm),
            conv=conv,
            z=_sparse_random(rng, (ZD, H), density, nrm),
            b=_sparse_random(rng, (NV, H), density, nrm),
            a=_sparse_random(rng, (NV, H), density, nrm),
            out=_sparse_random(rng, (H, ZD), density, nrm),
            A_log=bf16_bits(np.log(rng.uniform(0.0, 16.0, NV)).astype(np.float32)),
            dt_bias=bf16_bits(np.ones(NV, np.float32)),
            gnorm=bf16_bits(np.ones(VD, np.float32)),
            ln_in=np.zeros(H, np.uint16),
            ln_post=np.zeros(H, np.uint16),
            gate=_sparse_random(rng, (INTER, H), density, nrm),
            up=_sparse_random(rng, (INTER, H), density, nrm),
            down=_sparse_random(rng, (H, INTER), density, nrm),
        ))
    embed = bf16_bits(rng.normal(0.0, 0.02, (vocab, H)).astype(np.float32))
    head = _sparse_random(rng, (vocab, H), density, nrm)
    return Chip(name=f"c1(seed={seed},layers={n_layers},vocab={vocab},density={density})",
                layers=layers, embed=embed, head=head, final_norm=np.zeros(H, np.uint16),
                eps=1e-6, meta={"config": 1, "seed": seed})


def c1_state(chip: Chip, seed: int = 0, std: float = 1e-3) -> State:
    """Config 1's initial state: recurrent N(0, std) fp32, conv windows zero."""
    rng = np.random.default_rng(seed + 1_000_003)
    rec = rng.normal(0.0, std, (chip.n_layers, NV, KD, VD)).astype(np.float32)
    return State(rec, np.zeros((chip.n_layers, CONV, TAPS), np.uint16))


# --- the stock model (transformers), for the reference's own forward ----------------------------
def hf_config(chip: Chip):
    from transformers import Qwen3_5TextConfig

    n = chip.n_layers
    return Qwen3_5TextConfig(
        hidden_size=H, num_hidden_layers=n, layer_types=["linear_attention"] * n,
        vocab_size=chip.n_vocab, linear_key_head_dim=KD, linear_value_head_dim=VD,
        linear_num_key_heads=NK, linear_num_value_heads=NV, intermediate_size=INTER,
        linear_conv_kernel_dim=TAPS, hidden_act="silu", rms_norm_eps=chip.eps,
        tie_word_embeddings=False, num_attention_heads=16, num_key_value_heads=4, head_dim=256)


def to_hf(chip: Chip):
    """The chip as a stock Qwen3_5ForCausalLM (bf16, CPU): the model the reference's
    hf.chip_forward / hf.head_argmax run (lx/lx/hf.py:169-184)."""
    import torch
    from transformers import Qwen3_5ForCausalLM

    cfg = hf_config(chip)
    with torch.device("meta"):
        model = Qwen3_5ForCausalLM(cfg)

    def t(bits, shape=None):
        x = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)
        return x.reshape(shape) if shape is not None else x

    sd = {}
    for i, L in enumerate(chip.layers):
        p = f"model.layers.{i}."
        sd[p + "linear_attn.in_proj_qkv.weight"] = t(L.qkv.to_dense())
        sd[p + "linear_attn.conv1d.weight"] = t(L.conv, (CONV, 1, TAPS))
        sd[p + "linear_attn.in_proj_z.weight"] = t(L.z.to_dense())
        sd[p + "linear_attn.in_proj_b.weight"] = t(L.b.to_dense())
        sd[p + "linear_attn.in_proj_a.weight"] = t(L.a.to_dense())
        sd[p + "linear_attn.out_proj.weight"] = t(L.out.to_dense())
        sd[p + "linear_attn.A_log"] = t(L.A_log)
        sd[p + "linear_attn.dt_bias"] = t(L.dt_bias)
        sd[p + "linear_attn.norm.weight"] = t(L.gnorm)
        sd[p + "input_layernorm.weight"] = t(L.ln_in)
        sd[p + "post_attention_layernorm.weight"] = t(L.ln_post)
        sd[p + "mlp.gate_proj.weight"] = t(L.gate.to_dense())
        sd[p + "mlp.up_proj.weight"] = t(L.up.to_dense())
        sd[p + "mlp.down_proj.weight"] = t(L.down.to_dense())
    sd["model.embed_tokens.weight"] = t(chip.embed)
    sd["model.norm.weight"] = t(chip.final_norm)
    sd["lm_head.weight"] = t(chip.head.to_dense())
    missing, unexpected = model.load_state_dict(sd, strict=False, assign=True)
    assert not unexpected and not missing, (missing[:5], unexpected[:5])
    # the rotary tables are buffers, not weights: build them on the host so the model can move
    model.model.rotary_emb = type(model.model.rotary_emb)(config=cfg)
    return model.eval()


# --- config 2: the full 37-layer chip-shaped stack ------------------------------------------
C2_LAYERS = 37
C2_LOGIC = 15            # layers 0..14 carry the SwiGLU units; 15..36 are GDN-only (memory)
C2_HEADS = 497           # live key heads
C2_UNITS = 36716         # live SwiGLU units
C2_VOCAB = 459982
C2_RAM, C2_ROM = 4718592, 1009088
N_BALLAST, N_SEL = 8, 1024
SEL0 = N_BALLAST                      # select columns [8, 1032)
DATA0 = SEL0 + N_SEL                  # data columns [1032, 2560)
N_CODE = 31                           # the head's dense code columns: the last 31 data columns


def _pow2_values(rng, n):
    """values uniform in {-1, -0.5, 0.5, 1} x 2^k, k in [-4, 4] (all exact in bf16)."""
    m = rng.choice(np.array([-1.0, -0.5, 0.5, 1.0], np.float32), n)
    return (m * np.exp2(rng.integers(-4, 5, n)).astype(np.float32)).astype(np.float32)


def c2(seed: int = 1, vocab: int = C2_VOCAB, n_layers: int = C2_LAYERS) -> Chip:
    """Config 2: a 37-layer chip-shaped stack with the real circuit's sizes and a per-token
    activity shaped like the measured one (lx/results/summary.md:81: of the live value heads
    ~375 get a nonzero query or key, ~4.5 change state, ~21 produce output).

    Residual columns: 8 ballast columns (a constant 2.0 in every embedding row, never written,
    so every RMSNorm sees a stable scale), 1024 select columns (set by the embedding only), 1528
    data columns (embedding features, written by out_proj and down_proj). Every live key head
    reads its queries from one select column and its keys from another (one in_proj entry per
    channel, one conv tap on the newest input), so whether a head is active is decided by which
    select columns the current token sets: memory heads' queries fire for ~1.7% of tokens, the
    other heads' for ~13%, keys for ~0.15%. Value channels read 15 data columns each (every
    token, as in the real circuit, since their conv windows are state); only memory heads
    have in_proj_z rows. Query and key rows of
    the non-memory heads are disjoint, so only memory heads (whose states hold the RAM and ROM
    bytes, see c2_state) produce output. Layers 0..14 carry the 36,716 SwiGLU units (8 gate and
    8 up entries, one down weight each); layers 15..36 are GDN only, as the real circuit's
    last 22 layers. Two logic layers decay (dt_bias 1, in_proj_a entries); the rest have
    dt_bias -110 and empty in_proj_a rows, so their g is exactly 0. The head: 31 dense code
    columns with 2-bit codes over {-1/8, -1/16, 1/16, 1/8}. All weights are in
    {+-1, +-0.5} x 2^k, k in [-4, 4], drawn from `seed`."""
    rng = np.random.default_rng(seed)
    data_cols = np.arange(DATA0, H)
    heads_per_layer = np.full(n_layers, C2_HEADS // n_layers)
    heads_per_layer[:C2_HEADS - heads_per_layer.sum()] += 1
    n_logic = min(C2_LOGIC, n_layers)
    units_per_layer = np.zeros(n_layers, np.int64)
    units_per_layer[:n_logic] = C2_UNITS // n_logic
    units_per_layer[:C2_UNITS - units_per_layer.sum()] += 1
    decay_layers = {4, 9} & set(range(n_logic))
    sel_free = list(rng.permutation(N_SEL) + SEL0)
    meta = {"config": 2, "seed": seed, "memory_heads": [], "q_sel": {}, "k_sel": {}}
    layers = []
    mem_budget = -(-(C2_RAM // 15) // KD) + -(-(C2_ROM // 64) // KD)  # value heads of RAM+ROM
    mem_vh_left = mem_budget
    for L in range(n_layers):
        nkh = int(heads_per_layer[L])
        khs = np.sort(rng.choice(NK, nkh, replace=False))
        rows, cols, vals = [], [], []
        taps = np.zeros((CONV, TAPS), np.uint16)
        b_r, b_c, a_r, a_c, z_r, z_c, o_r, o_c = [], [], [], [], [], [], [], []
        decays = L in decay_layers
        for kh in khs:
            memory = L >= n_logic and mem_vh_left > 0
            if memory:
                mem_vh_left -= R
                meta["memory_heads"].append((L, int(kh)))
            qs, ks = sel_free.pop(), sel_free.pop()
            meta["q_sel"][(L, int(kh))] = qs
            meta["k_sel"][(L, int(kh))] = ks
            qrows = rng.choice(KD, 8, replace=False)
            krows = qrows if memory else rng.choice(np.setdiff1d(np.arange(KD), qrows), 8,
                                                    replace=False)
            for base, rr, sc in ((kh * KD, qrows, qs), (NK * KD + kh * KD, krows, ks)):
                ch = base + rr
                rows.append(ch)
                cols.append(np.full(len(ch), sc))
                vals.append(_pow2_values(rng, len(ch)))
                taps[ch, 3] = bf16_bits(_pow2_values(rng, len(ch)))
            vch = 2 * NK * KD + kh * R * VD + rng.choice(R * VD, 700, replace=False)
            rows.append(np.repeat(vch, 15))
            cols.append(rng.integers(DATA0, H, len(vch) * 15))
            vals.append(_pow2_values(rng, len(vch) * 15))
            single = rng.random(len(vch)) < 0.8
            taps[vch[single], 3] = bf16_bits(_pow2_values(rng, int(single.sum())))
            multi = vch[~single]
            taps[multi] = bf16_bits(_pow2_values(rng, len(multi) * TAPS)).reshape(-1, TAPS)
            vh = kh * R + np.arange(R)
            for v in vh:
                b_r.append(np.full(4, v))
                b_c.append(rng.choice(data_cols, 4, replace=False))
                if decays:
                    a_r.append(np.full(2, v))
                    a_c.append(rng.choice(data_cols, 2, replace=False))
            dims = (vh[:, None] * VD + np.arange(VD)).reshape(-1)
            if memory:  # only memory heads can produce output
                z_r.append(dims)
                z_c.append(rng.choice(data_cols, len(dims)))
                od = rng.choice(dims, 330, replace=False)
                o_r.append(rng.choice(data_cols, len(od)))
                o_c.append(od)
        cat = lambda x: np.concatenate(x) if x else np.zeros(0, np.int64)  # noqa: E731
        qkv = Sparse.from_coo((CONV, H), cat(rows), cat(cols), bf16_bits(cat(vals)))
        mk = lambda r, c, shape: Sparse.from_coo(shape, cat(r), cat(c), bf16_bits(  # noqa: E731
            _pow2_values(rng, len(cat(r)))))
        nu = int(units_per_layer[L])
        if nu:
            u = np.sort(rng.choice(INTER, nu, replace=False))
            gr, gc = np.repeat(u, 8), rng.choice(data_cols, nu * 8)
            gate = Sparse.from_coo((INTER, H), gr, gc, bf16_bits(_pow2_values(rng, nu * 8)))
            up = Sparse.from_coo((INTER, H), gr, rng.choice(data_cols, nu * 8),
                                 bf16_bits(_pow2_values(rng, nu * 8)))
            down = Sparse.from_coo((H, INTER), rng.choice(data_cols, nu), u,
                                   bf16_bits(_pow2_values(rng, nu)))
        else:
            gate = up = Sparse.from_coo((INTER, H), [], [], [])
            down = Sparse.from_coo((H, INTER), [], [], [])
        layers.append(Layer(
            qkv=qkv, conv=taps,
            z=mk(z_r, z_c, (ZD, H)),
            b=mk(b_r, b_c, (NV, H)),
            a=mk(a_r, a_c, (NV, H)),
            out=mk(o_r, o_c, (H, ZD)),
            A_log=np.zeros(NV, np.uint16),  # A = -exp(0) = -1
            dt_bias=bf16_bits(np.where(np.isin(np.arange(NV) // R, khs) & decays, 1.0,
                                       -110.0).astype(np.float32)),
            gnorm=bf16_bits(np.ones(VD, np.float32)),
            ln_in=np.zeros(H, np.uint16), ln_post=np.zeros(H, np.uint16),
            gate=gate, up=up, down=down))
    # the embedding: ballast, select columns by head kind, ~48 data features
    emb = np.zeros((vocab, H), np.uint16)
    emb[:, :N_BALLAST] = bf16_bits(np.float32(2.0))
    mem = set(meta["memory_heads"])
    for (L, kh), qs in meta["q_sel"].items():
        p = 0.017 if (L, kh) in mem else 0.13
        on = np.nonzero(rng.random(vocab) < p)[0]
        emb[on, qs] = bf16_bits(_pow2_values(rng, len(on)))
    for (L, kh), ks in meta["k_sel"].items():
        on = np.nonzero(rng.random(vocab) < 0.0015)[0]
        emb[on, ks] = bf16_bits(_pow2_values(rng, len(on)))
    nf = 48
    fr = np.repeat(np.arange(vocab), nf)
    fc = rng.integers(DATA0, H - N_CODE, vocab * nf)
    emb[fr, fc] = bf16_bits(rng.choice(np.array([-1.0, 1.0], np.float32), vocab * nf))
    # every token carries a +-1 pattern in the code columns (the head reads them back)
    emb[:, H - N_CODE:] = bf16_bits(rng.choice(np.array([-1.0, 1.0], np.float32),
                                               (vocab, N_CODE)))
    # the head: 31 dense code columns, 2-bit codes
    code_cols = np.arange(H - N_CODE, H)
    hv = np.array([-0.125, -0.0625, 0.0625, 0.125], np.float32)
    codes = rng.integers(0, 4, (vocab, N_CODE))
    head = Sparse((vocab, H), np.arange(vocab + 1, dtype=np.int64) * N_CODE,
                  np.tile(code_cols.astype(np.int32), vocab), bf16_bits(hv[codes]).reshape(-1))
    meta["memory_value_heads"] = (mem_budget - mem_vh_left)
    meta["q_sel"] = {f"{k[0]}.{k[1]}": int(v) for k, v in meta["q_sel"].items()}
    meta["k_sel"] = {f"{k[0]}.{k[1]}": int(v) for k, v in meta["k_sel"].items()}
    return Chip(name=f"c2(seed={seed},layers={n_layers},vocab={vocab})", layers=layers,
                embed=emb, head=head, final_norm=np.zeros(H, np.uint16), eps=1e-6, meta=meta)


def c2_state(chip: Chip, seed: int = 1) -> State:
    """Config 2's initial state: 5.5 MB of uniform random bytes in the memory heads' rows.
    RAM (4,718,592 bytes): 15 bytes per state row as 120 bit columns (0 or 128) in columns
    2..121, with ballast 2^24 in columns 0 and 1; ROM (1,009,088 bytes): 64 bytes per row as 128
    nibble columns (integers 0..15). Filled in order over the memory heads' value heads."""
    rng = np.random.default_rng(seed + 7_000_003)
    L_n = chip.n_layers
    rec = np.zeros((L_n, NV, KD, VD), np.float32)
    ram = rng.integers(0, 256, C2_RAM, dtype=np.uint8)
    rom = rng.integers(0, 256, C2_ROM, dtype=np.uint8)
    ram_rows = -(-C2_RAM // 15)
    rbuf = np.zeros(ram_rows * 15, np.uint8)
    rbuf[:C2_RAM] = ram
    bits = np.unpackbits(rbuf.reshape(ram_rows, 15), axis=1)            # [rows, 120]
    ram_f = np.zeros((ram_rows, VD), np.float32)
    ram_f[:, 0:2] = 2.0 ** 24
    ram_f[:, 2:122] = bits * 128.0
    rom_rows = -(-C2_ROM // 64)
    obuf = np.zeros(rom_rows * 64, np.uint8)
    obuf[:C2_ROM] = rom
    nib = np.stack([obuf >> 4, obuf & 15], 1).reshape(rom_rows, VD).astype(np.float32)
    all_rows = np.concatenate([ram_f, nib])
    vhs = [(L, kh * R + r) for (L, kh) in chip.meta["memory_heads"] for r in range(R)]
    k = 0
    for L, vh in vhs:
        if k >= len(all_rows):
            break
        n = min(KD, len(all_rows) - k)
        rec[L, vh, :n] = all_rows[k:k + n]
        k += n
    return State(rec, np.zeros((L_n, CONV, TAPS), np.uint16))


# --- the real compiled circuit (a fixture made by the reference's own compiler) -----------------
# (file key, the stock layer's weight name) of every projection / per-head vector in the fixture
REAL_MATS = (("qkv", "linear_attn.in_proj_qkv.weight"), ("z", "linear_attn.in_proj_z.weight"),
             ("b", "linear_attn.in_proj_b.weight"), ("a", "linear_attn.in_proj_a.weight"),
             ("out", "linear_attn.out_proj.weight"), ("gate", "mlp.gate_proj.weight"),
             ("up", "mlp.up_proj.weight"), ("down", "mlp.down_proj.weight"))
REAL_VECS = (("A_log", "linear_attn.A_log"), ("dt_bias", "linear_attn.dt_bias"),
             ("gnorm", "linear_attn.norm.weight"), ("ln_in", "input_layernorm.weight"),
             ("ln_post", "post_attention_layernorm.weight"))


def real_path():
    from pathlib import Path

    return Path(__file__).resolve().parents[1] / "tests" / "golden" / "real_chip.npz"


def real(path=None, vocab: int | None = None) -> Chip:
    """The real circuit's chip layers (the reference's compiler, ``lx.core.build(merge.config())``
    emitted at hidden 2560 as the merged model has them, lx/lx/merge.py:123-157), the chip
    vocabulary's embedding rows and, tied to them, the head (lx/lx/hf.py:63-93); final norm weight
    0. ``vocab`` keeps only the first head rows (tests). The fixture's machine (program, RAM
    seed, the RAM/ROM placement, the other tables' rows) and the reference machine's trace ride
    along in ``meta``; ``real_state`` builds the state. Made by tests/golden/make_real.py."""
    import json

    z = np.load(path or real_path())
    meta = json.loads(bytes(z["meta"]).decode())
    layers = []
    for L in range(meta["n_layers"]):
        mats = {}
        for f, _ in REAL_MATS:
            cnt = z[f"L{L}.{f}.cnt"]
            indptr = np.zeros(len(cnt) + 1, np.int64)
            np.cumsum(cnt, out=indptr[1:])
            shape = {"qkv": (CONV, H), "z": (ZD, H), "b": (NV, H), "a": (NV, H),
                     "out": (H, ZD), "gate": (INTER, H), "up": (INTER, H), "down": (H, INTER)}[f]
            assert len(cnt) == shape[0]
            mats[f] = Sparse(shape, indptr, z[f"L{L}.{f}.idx"].astype(np.int32),
                             z[f"L{L}.{f}.val"].astype(np.uint16))
        vecs = {f: z[f"L{L}.{f}"].astype(np.uint16) for f, _ in REAL_VECS}
        layers.append(Layer(conv=z[f"L{L}.conv"].astype(np.uint16), **mats, **vecs))
    cols = z["emb_cols"].astype(np.int64)
    vals = z["emb_vals"]
    emb = np.zeros((vals.shape[0], H), np.uint16)
    emb[:, cols] = vals
    V = meta["vocab"] if vocab is None else vocab
    r, k = np.nonzero(vals[:V] & 0x7FFF)
    head = Sparse.from_coo((V, H), r, cols[k], vals[r, k])
    fix = {k: z[k] for k in ("ram_map", "rom_map", "init_idx", "init_rows", "program", "trace")}
    meta = dict(meta, config="real", fixture=fix)
    return Chip(name="real circuit (merged config)" + (f", vocab={vocab}" if vocab else ""),
                layers=layers, embed=emb, head=head, final_norm=np.zeros(H, np.uint16),
                eps=float(meta["eps"]), meta=meta)


def real_ram(chip: Chip) -> np.ndarray:
    """The fixture machine's RAM bytes: seeded uniform random bytes, the program at the reset
    address (checked against the fixture's digest)."""
    m = chip.meta
    ram = np.random.default_rng(m["ram_seed"]).integers(0, 256, m["ram_size"], dtype=np.uint8)
    prog = m["fixture"]["program"]
    ram[:len(prog)] = prog
    assert hashlib.sha256(ram.tobytes()).hexdigest() == m["ram_sha256"], "RAM bytes"
    return ram


def real_state(chip: Chip, ram: np.ndarray | None = None) -> State:
    """The machine's state in the GDN states, placed as the reference's ``lx.core.snapshot`` and
    ``lx.hf.inject`` place it (lx/lx/core.py:1343-1414, lx/lx/hf.py:154-166):

    - RAM block b (2048 words) lives in the value heads of key head j of layer L (the fixture's
      map): word i of the block, if nonzero, is row i >> 3 of value head j * 8 + (i & 7): the
      ballast a_ref in columns 0 and 1 and a_bit in column 2 + k for each set bit k;
    - ROM head h (the first text_words words, 16384 a head): value head x of its key head holds
      words [2048 x, 2048 (x + 1)) of the head's range, 8 words a row, the ballast in columns
      0 and 1 and word k's 8 nibbles (low first) in columns 2 + 8 k ..;
    - every other table's rows verbatim from the fixture.
    Conv windows start at zero (a fresh session runs one zero step first, which leaves them so)."""
    m, fx = chip.meta, chip.meta["fixture"]
    ram = real_ram(chip) if ram is None else ram
    rec = np.zeros((chip.n_layers, NV, KD, VD), np.float32)
    a_ref, a_bit, rw = np.float32(m["a_ref"]), np.float32(m["a_bit"]), m["ram_head_words"]
    refc = list(m["ref_cols"])
    words = ram.view("<u4")
    bitk = np.arange(32, dtype=np.uint32)
    for blk, L, j in fx["ram_map"]:
        seg = words[blk * rw:(blk + 1) * rw]
        wi = np.nonzero(seg)[0]
        rows = np.zeros((len(wi), VD), np.float32)
        rows[:, refc] = a_ref
        rows[:, 2:34] = ((seg[wi, None] >> bitk) & 1).astype(np.float32) * a_bit
        rec[L, j * R + (wi & 7), wi >> 3] = rows
    rom = words[:m["text_words"]]
    hw = m["rom_head_words"]
    nib = np.arange(8, dtype=np.uint32) * 4
    for h, L, j in fx["rom_map"]:
        for x in range(R):
            base = h * hw + x * rw
            blk = rom[base:base + rw] if base < len(rom) else rom[:0]
            nr = -(-len(blk) // 8)
            if nr == 0:
                continue
            pad = np.zeros(nr * 8, np.uint32)
            pad[:len(blk)] = blk
            rows = np.zeros((nr, VD), np.float32)
            rows[:, refc] = a_ref
            rows[:, 2:66] = ((pad.reshape(nr, 8)[:, :, None] >> nib) & 15).reshape(nr, 64)
            rec[L, j * R + x, :nr] = rows
    ii = fx["init_idx"]
    rec[ii[:, 0], ii[:, 1], ii[:, 2]] = fx["init_rows"]
    return State(rec, np.zeros((chip.n_layers, CONV, TAPS), np.uint16))
