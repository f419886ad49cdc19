"""The quantized ResNet-18 restated with the oracle's functions (test infrastructure): the
same f32 parameters and the activation scales a device run calibrated, layer by layer --
quantize_value / find_scale_zp (quantization/helpers.rs:101-160), BN folding
(ir/optimizer.rs:727-731), per-channel INT8 weights, the INT8 chain (cpu/quantized_ops.rs:13-48)
as direct int8 convolutions, int8 max / average pools (operator/pooling.rs:383-530)."""
import numpy as np

from oracle import oracle as orc


def oracle_resnet18(x, model, rounding):
    """The quantized network restated with the oracle's functions."""
    sc = model.scales
    xq = orc.quantize_nchw_to_nhwc(x, sc["input"], 16, rounding)
    acts = {"x_q": xq}

    def conv(spec, in_name, residual=None):
        xin = acts[in_name]
        s_in = sc["input"] if in_name == "x_q" else sc[in_name]
        wf, bf = orc.bn_fold(spec.w, spec.bias, *spec.bn)
        wq, sw = orc.quantize_weights_per_channel(np.ascontiguousarray(wf.transpose(0, 2, 3, 1)))
        cs = xin.shape[3]
        wp = np.zeros((spec.cout, spec.k, spec.k, cs), np.int8)
        wp[..., :spec.cin] = wq
        scale = (np.float32(s_in) * sw).astype(np.float32)
        bq = np.array([orc.quantize_value(float(bf[o]), float(scale[o]), 0, orc.QINT32) for o in range(spec.cout)],
                      np.int32)
        res = None if residual is None else acts[residual]
        rs = 1.0 if residual is None else sc[residual]
        q, _, _ = orc.conv2d_i8_nhwc_chain(xin, wp, bq, scale, (spec.stride,) * 2, (spec.pad,) * 2, (1, 1), 1,
                                           orc.ACT_RELU if spec.relu else orc.ACT_NONE, sc[spec.name], rounding,
                                           residual=res, residual_scale=rs)
        acts[spec.name] = q

    conv(model.convs[0], "x_q")
    acts["pool"] = orc.maxpool_i8_nhwc(acts["conv1"], 3, 2, 1)
    sc = dict(sc)
    prev = "pool"
    for c1, c2, ds in model.blocks:
        conv(c1, prev)
        if ds is not None:
            conv(ds, prev)
            res = ds.name
        else:
            res = prev
        conv(c2, c1.name, residual=res)
        prev = c2.name
    pooled, _ = orc.avgpool_i8_nhwc(acts[prev], sc[prev], sc["pooled"], rounding)
    wq, sw = orc.quantize_weights_per_channel(model.fc_w)
    scale = (np.float32(sc["pooled"]) * sw).astype(np.float32)
    bq = np.array([orc.quantize_value(float(model.fc_b[o]), float(scale[o]), 0, orc.QINT32)
                   for o in range(model.num_classes)], np.int32)
    _, logits, _ = orc.gemm_i8_chain(pooled, wq, bq, scale, orc.ACT_NONE, 1.0, rounding)
    return logits, acts
