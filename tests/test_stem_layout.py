"""CPU restatement of the one-launch ResNet stem's index logic (lightship_b200/csrc/stem_i8.cu),
checked against direct definitions on small cases, without a GPU:

- the conv-row sequence a CTA walks (its pooled rows, plus the row above the first one) covers
  every pooled row once, and each pooled row finds its three conv rows where the epilogue reads
  them;
- the input loads (two rows x three channels each, slot = count mod 12, four conv rows ahead)
  never overwrite a slot that is still to be read, and the 16-row ring of quantized rows holds
  the seven input rows of every conv row's window when its im2col rows are built, untouched by
  the quantization of the next conv row;
- the four shifted copies of a quantized row (built from words u, u+1, u+2 with funnel shifts)
  and the 8-byte gather per (channel, kh) group, with the filter image's K order and
  core-matrix layout, reproduce the direct 7x7 / 2 convolution (int32);
- the epilogue's lane / column mapping (channels on TMEM lanes, pixel x at column x + 4, four
  column slices of 14 pooled columns) reproduces the 3x3 / 2 max pool with padding taps
  skipped, including pooling the accumulators before requantization.
"""
import numpy as np

PH = 56          # pooled rows per image
LEAD, SLOTS, RING = 4, 12, 16


def stem_item(i, g0, e):
    if e and i == 0:
        n = g0 // PH
        return n, 2 * (g0 - n * PH) - 1, 1
    j = i - e
    g = g0 + (j >> 1)
    n = g // PH
    r = 2 * (g - n * PH) + (j & 1)
    return n, r, 1 if (i == 0 or r == 0) else 0


def loads(it):
    return 4 if it[2] else 1


def new_rows(it):
    return 7 if it[2] else 2


def first_row(it):
    return 2 * it[1] - 3 if it[2] else 2 * it[1] + 2


def _check_cta(g0, g1):
    e = 1 if g0 % PH else 0
    items = 2 * (g1 - g0) + e
    seq = [stem_item(i, g0, e) for i in range(items)]
    # pooled rows and the conv rows the epilogue reads for them
    for gi in range(g0, g1):
        n, py = divmod(gi, PH)
        il = e + 2 * (gi - g0) + 1
        assert seq[il][:2] == (n, 2 * py + 1) and seq[il - 1][:2] == (n, 2 * py)
        if py > 0:
            assert seq[il - 2][:2] == (n, 2 * py - 1)
    # loads, slots and the quantized ring, in the builders' order
    L = [(k, it[0], first_row(it) + 2 * j) for k, it in enumerate(seq) for j in range(loads(it))]
    slot_of, ring = {}, {}
    state = {"issued": 0, "used": 0, "q": 0}

    def issue_upto(upto):
        while state["issued"] < len(L) and L[state["issued"]][0] <= upto:
            s = state["issued"] % SLOTS
            assert s not in slot_of or slot_of[s] < state["used"], "a load overwrites an unread slot"
            slot_of[s] = state["issued"]
            state["issued"] += 1

    def quantize(k):
        it = seq[k]
        for ri in range(new_rows(it)):
            li = state["used"] + (ri >> 1)
            assert slot_of[li % SLOTS] == li
            assert L[li][1] == it[0] and L[li][2] + (ri & 1) == first_row(it) + ri
            ring[(state["q"] + ri) % RING] = (it[0], first_row(it) + ri)
        state["used"] += loads(it)
        state["q"] += new_rows(it)

    issue_upto(LEAD)
    quantize(0)
    for i in range(items):
        issue_upto(i + LEAD + 1)
        n, r, _ = seq[i]
        q = state["q"]
        for kh in range(7):
            assert ring[(q - 7 + kh) % RING] == (n, 2 * r - 3 + kh)
        if i + 1 < items:
            written = {(q + x) % RING for x in range(new_rows(seq[i + 1]))}
            assert not written & {(q - 7 + x) % RING for x in range(7)}
            quantize(i + 1)
    return items


def test_cta_sequences_cover_every_pooled_row_and_keep_their_inputs():
    for nimg, sms in [(1, 1), (1, 56), (2, 3), (3, 5), (4, 148), (5, 148), (7, 13), (32, 148), (85, 148),
                      (256, 148)]:
        G = nimg * PH
        grid = min(sms, G)
        covered = np.zeros(G, int)
        for b in range(grid):
            g0, g1 = b * G // grid, (b + 1) * G // grid
            assert g1 > g0
            _check_cta(g0, g1)
            covered[g0:g1] += 1
        assert (covered == 1).all()


def _filter_image(ws2d):
    img = np.zeros(12288, np.int8)
    for co in range(64):
        for c in range(3):
            for kh in range(7):
                for kw in range(7):
                    k = 8 * (c * 7 + kh) + kw
                    img[(k // 16) * 1024 + (co // 8) * 128 + (co % 8) * 16 + (k % 16)] = \
                        ws2d[co, kh // 2, kw // 2, ((kh % 2) * 2 + kw % 2) * 3 + c]
    return img


def _copies(P):
    """The four copies of row image P shifted by 1, 3, 5, 7 bytes, as the warp builds them."""
    pw = P.view(np.uint32).astype(np.uint64)
    out = np.zeros((4, 288), np.uint8)
    for u in range(62):
        a, b, d = int(pw[u]), int(pw[u + 1]), int(pw[u + 2])
        ab, bd = (b << 32) | a, (d << 32) | b
        for k, v in enumerate([(ab >> 8), (ab >> 24), (bd >> 8), (bd >> 24)]):
            out[k, 4 * u:4 * u + 4] = np.frombuffer(np.uint32(v & 0xFFFFFFFF).tobytes(), np.uint8)
    return out


def test_im2col_gather_and_filter_image_give_the_direct_convolution():
    rng = np.random.default_rng(3)
    xq = rng.integers(-128, 128, size=(3, 224, 224)).astype(np.int64)
    w7 = rng.integers(-127, 128, size=(64, 3, 7, 7)).astype(np.int8)
    ws2d = np.zeros((64, 4, 4, 16), np.int8)
    for co in range(64):
        for c in range(3):
            for kh in range(7):
                for kw in range(7):
                    ws2d[co, kh // 2, kw // 2, ((kh % 2) * 2 + kw % 2) * 3 + c] = w7[co, c, kh, kw]
    img = _filter_image(ws2d)
    W = np.array([[img[(k // 16) * 1024 + (co // 8) * 128 + (co % 8) * 16 + (k % 16)] for k in range(192)]
                  for co in range(64)], np.int64)
    xp = np.zeros((3, 230, 230), np.int64)
    xp[:, 3:227, 3:227] = xq
    copies = {}
    for c in range(3):
        for iy in range(-3, 226):
            P = np.zeros(256, np.uint8)
            if 0 <= iy < 224:
                P[8:232] = (xq[c, iy] & 0xFF).astype(np.uint8)   # P[i] = q(x[i - 8])
            copies[(c, iy)] = _copies(P)
    for r in [0, 1, 54, 110, 111]:
        conv = np.zeros((112, 64), np.int64)
        for kh in range(7):
            for kw in range(7):
                conv += xp[:, 2 * r + kh, kw:kw + 224:2].T @ w7[:, :, kh, kw].T.astype(np.int64)
        B = np.zeros((112, 192), np.int64)
        for x in range(112):
            o = 2 * x + 5
            k, j = (o & 7) >> 1, o & ~7
            for q in range(21):
                c, kh = divmod(q, 7)
                B[x, 8 * q:8 * q + 8] = copies[(c, 2 * r - 3 + kh)][k, j:j + 8].view(np.int8)
        np.testing.assert_array_equal(B @ W.T, conv)


def test_epilogue_mapping_is_the_max_pool_and_commutes_with_requantization():
    rng = np.random.default_rng(4)
    conv = rng.integers(-2 ** 21, 2 ** 21, size=(112, 112, 64))
    blocks = {}
    for r in range(112):          # TMEM block: lanes = channels, column x + 4; garbage elsewhere
        b = rng.integers(-2 ** 30, 2 ** 30, size=(64, 128))
        b[:, 4:116] = conv[r].T
        blocks[r] = b
    got = np.zeros((56, 56, 64), np.int64)
    for py in range(56):
        for sl in range(4):
            cols = 28 * sl + np.arange(32)
            m = np.maximum(blocks[2 * py + 1][:, cols], blocks[2 * py][:, cols])
            if py > 0:
                m = np.maximum(m, blocks[2 * py - 1][:, cols])
            for j in range(14):
                v = m[:, 2 * j + 3:2 * j + 6].max(axis=1)
                if j == 0 and sl == 0:
                    v = m[:, 4:6].max(axis=1)
                got[py, 14 * sl + j] = v
    want = np.full((56, 56, 64), np.iinfo(np.int64).min)
    for py in range(56):
        for px in range(56):
            for yy in range(max(2 * py - 1, 0), min(2 * py + 2, 112)):
                for xx in range(max(2 * px - 1, 0), min(2 * px + 2, 112)):
                    want[py, px] = np.maximum(want[py, px], conv[yy, xx])
    np.testing.assert_array_equal(got, want)
    # requantization (bias, positive scale, ReLU, round half even, saturate) is monotone, so
    # pooling the accumulators first gives the same codes as pooling the codes
    bias = rng.integers(-5000, 5000, size=64)
    scale = rng.uniform(1e-4, 1e-3, size=64).astype(np.float32)

    def requant(a):
        y = (a + bias).astype(np.float32) * scale
        return np.clip(np.rint(np.maximum(y, 0) / np.float32(0.05)), -128, 127).astype(np.int8)

    codes = requant(conv)
    pooled_codes = np.full((56, 56, 64), -128, np.int8)
    for py in range(56):
        for px in range(56):
            win = codes[max(2 * py - 1, 0):2 * py + 2, max(2 * px - 1, 0):2 * px + 2]
            pooled_codes[py, px] = win.reshape(-1, 64).max(axis=0)
    np.testing.assert_array_equal(requant(got), pooled_codes)
