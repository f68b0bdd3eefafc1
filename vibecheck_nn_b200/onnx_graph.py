"""ONNX networks for the B200 path without the ``onnx`` package.

* ``read_onnx(path)`` decodes the ONNX protobuf wire format (ModelProto ->
  GraphProto -> NodeProto / TensorProto / AttributeProto / ValueInfoProto,
  the field numbers of the published onnx.proto) into an ``OnnxGraph``.
* ``OnnxGraph.to_gg(device, dtype)`` builds the op dict the reference's
  loader and ``ComputeGraph.gpu_graph`` produce for fc / ReLU networks
  (onnx_loader.py:12-604, network.py:1707-2910): MatMul and Gemm become
  ``fc`` ops (weights (out, in), MatMul with a zero bias), an Add or Sub of
  a constant becomes an ``add`` / ``sub`` op carrying it, Mul / Div by a
  constant a ``mul`` op, Flatten / Reshape a ``reshape`` passthrough, Relu a
  ``relu`` with its layer index; constant-only subgraphs are folded.
* ``OnnxGraph.forward64(x)`` evaluates the network in float64 on the host:
  the replay that confirms a SAT witness (in place of the reference's
  onnxruntime replay, verify_graph.py:5423-5467).

Other operators raise ``UnsupportedInput``.
"""
from __future__ import annotations

import gzip
import struct

import numpy as np

from . import _lib

# TensorProto.DataType values used by fc / ReLU networks
_DTYPES = {1: np.float32, 6: np.int32, 7: np.int64, 11: np.float64}


def _varint(b, i):
    r = s = 0
    while True:
        c = b[i]
        i += 1
        r |= (c & 0x7F) << s
        s += 7
        if not c & 0x80:
            return r, i


def _fields(b):
    """(field number, wire type, value) of one protobuf message: varints as
    ints, 64- and 32-bit fields as raw bytes, length-delimited as bytes."""
    i, n, out = 0, len(b), []
    while i < n:
        key, i = _varint(b, i)
        f, wt = key >> 3, key & 7
        if wt == 0:
            v, i = _varint(b, i)
        elif wt == 1:
            v, i = b[i:i + 8], i + 8
        elif wt == 2:
            ln, i = _varint(b, i)
            v, i = b[i:i + ln], i + ln
        elif wt == 5:
            v, i = b[i:i + 4], i + 4
        else:
            raise ValueError(f'protobuf wire type {wt} is not supported')
        out.append((f, wt, v))
    return out


def _packed_varints(v):
    out, i = [], 0
    while i < len(v):
        x, i = _varint(v, i)
        out.append(x)
    return out


def _int64(x):
    return x - (1 << 64) if x >= 1 << 63 else x


def _tensor(b):
    """TensorProto -> (name, numpy array)."""
    dims, dtype, name, raw = [], 1, '', None
    floats, doubles, ints = [], [], []
    for f, wt, v in _fields(b):
        if f == 1:
            dims.extend(_int64(x) for x in (_packed_varints(v) if wt == 2 else [v]))
        elif f == 2:
            dtype = v
        elif f == 8:
            name = v.decode()
        elif f == 9:
            raw = v
        elif f == 4:
            floats.extend(struct.unpack(f'<{len(v) // 4}f', v) if wt == 2 else
                          struct.unpack('<f', v))
        elif f == 10:
            doubles.extend(struct.unpack(f'<{len(v) // 8}d', v) if wt == 2 else
                           struct.unpack('<d', v))
        elif f in (5, 7):
            ints.extend(_int64(x) for x in (_packed_varints(v) if wt == 2 else [v]))
    if dtype not in _DTYPES:
        raise _lib.UnsupportedInput(f'vibecheck_nn_b200: ONNX tensor {name!r} dtype {dtype}')
    npt = _DTYPES[dtype]
    if raw is not None:
        arr = np.frombuffer(raw, dtype=np.dtype(npt).newbyteorder('<')).astype(npt)
    elif dtype == 1:
        arr = np.asarray(floats, np.float32)
    elif dtype == 11:
        arr = np.asarray(doubles, np.float64)
    else:
        arr = np.asarray(ints, npt)
    return name, arr.reshape(dims) if dims else arr.reshape(())


def _attribute(b):
    name, val, ints, floats = '', None, [], []
    for f, wt, v in _fields(b):
        if f == 1:
            name = v.decode()
        elif f == 2:
            val = struct.unpack('<f', v)[0]
        elif f == 3:
            val = _int64(v)
        elif f == 4:
            val = v.decode(errors='replace')
        elif f == 5:
            val = _tensor(v)[1]
        elif f == 7:
            floats.extend(struct.unpack(f'<{len(v) // 4}f', v) if wt == 2 else
                          struct.unpack('<f', v))
        elif f == 8:
            ints.extend(_int64(x) for x in (_packed_varints(v) if wt == 2 else [v]))
    if ints:
        val = ints
    elif floats:
        val = floats
    return name, val


def _value_info(b):
    name, dims = '', []
    for f, _, v in _fields(b):
        if f == 1:
            name = v.decode()
        elif f == 2:  # TypeProto
            for tf, _, tv in _fields(v):
                if tf != 1:  # tensor_type
                    continue
                for sf, _, sv in _fields(tv):
                    if sf != 2:  # shape
                        continue
                    for df, _, dv in _fields(sv):
                        if df == 1:  # dim
                            d = 0
                            for xf, xwt, xv in _fields(dv):
                                if xf == 1 and xwt == 0:
                                    d = _int64(xv)
                            dims.append(d)
    return name, dims


class OnnxGraph:
    """Nodes in file order (op_type, inputs, outputs, attributes), the
    initialisers and Constant outputs (float tensors promoted to float64, as
    the reference's loader does), the graph input's name and dims and the
    output name."""

    def __init__(self, nodes, consts, input_name, input_dims, output_name):
        self.nodes = nodes
        self.consts = consts
        self.input_name = input_name
        self.input_dims = input_dims
        self.output_name = output_name

    @property
    def input_shape(self):
        """The reference's resolved input shape: dims as given when all are
        concrete, else batch 1 followed by the data dims."""
        dims = self.input_dims
        conc = [d > 0 for d in dims]
        if all(conc):
            return tuple(dims)
        first = 1
        while first < len(dims) and not conc[first]:
            first += 1
        if first >= len(dims):
            return (1, dims[-1] if dims and dims[-1] > 0 else 1)
        return tuple([1] + [d if d > 0 else 1 for d in dims[first:]])

    @property
    def input_n(self):
        return int(np.prod([d for d in self.input_shape]))

    # ------------------------------------------------------------ lowering
    def _const(self, name):
        return self.consts.get(name)

    def to_gg(self, device, dtype):
        """The reference's gpu_graph op dict of this network (fc / relu /
        add / sub / mul / reshape ops)."""
        import torch
        ops, relu_names = [], []
        computed = {self.input_name}
        alias = {}
        consts = dict(self.consts)

        def src(n):
            return alias.get(n, n)

        def live(n):
            return src(n) in computed

        for op_type, ins, outs, attrs in self.nodes:
            name = outs[0]
            c = [consts.get(i) for i in ins]
            if op_type == 'Constant':
                continue
            if ins and all(x is not None for x in c):  # constant-only: fold
                consts[name] = _eval(op_type, c, attrs)
                continue
            if op_type in ('Identity', 'Dropout', 'Cast'):
                alias[name] = src(ins[0])
                continue
            if op_type in ('Flatten', 'Reshape'):
                ops.append({'name': name, 'type': 'reshape', 'inputs': [src(ins[0])]})
            elif op_type in ('MatMul', 'Gemm'):
                if op_type == 'MatMul':
                    if c[1] is None or c[0] is not None or c[1].ndim != 2:
                        raise _lib.UnsupportedInput(
                            f'vibecheck_nn_b200: MatMul {name!r} needs a constant 2-D weight')
                    W = c[1].T
                    b = np.zeros(W.shape[0])
                else:
                    if c[1] is None:
                        raise _lib.UnsupportedInput(
                            f'vibecheck_nn_b200: Gemm {name!r} with a non-constant weight')
                    if attrs.get('transA', 0) or attrs.get('alpha', 1.0) != 1.0 or \
                            attrs.get('beta', 1.0) != 1.0:
                        raise _lib.UnsupportedInput(
                            f'vibecheck_nn_b200: Gemm {name!r} with transA / alpha / beta')
                    W = c[1] if attrs.get('transB', 0) else c[1].T
                    b = c[2] if len(c) > 2 and c[2] is not None else np.zeros(W.shape[0])
                W = np.asarray(W, np.float64)
                b = np.asarray(b, np.float64).reshape(-1)
                ops.append({'name': name, 'type': 'fc', 'inputs': [src(ins[0])],
                            'W': torch.tensor(W, dtype=dtype, device=device),
                            'bias': torch.tensor(b, dtype=dtype, device=device),
                            'W_np': W, 'bias_np': b})
            elif op_type == 'Relu':
                ops.append({'name': name, 'type': 'relu', 'inputs': [src(ins[0])],
                            'layer_idx': len(relu_names)})
                relu_names.append(name)
            elif op_type in ('Add', 'Sub'):
                if live(ins[0]) and c[1] is not None:
                    ops.append({'name': name, 'type': 'add' if op_type == 'Add' else 'sub',
                                'inputs': [src(ins[0])], 'is_merge': False,
                                'bias': np.asarray(c[1], np.float64).reshape(-1)})
                elif op_type == 'Add' and live(ins[1]) and c[0] is not None:
                    ops.append({'name': name, 'type': 'add', 'inputs': [src(ins[1])],
                                'is_merge': False,
                                'bias': np.asarray(c[0], np.float64).reshape(-1)})
                else:
                    raise _lib.UnsupportedInput(
                        f'vibecheck_nn_b200: {op_type} {name!r} of two computed tensors')
            elif op_type in ('Mul', 'Div'):
                k = 1 if c[1] is not None else 0
                if c[k] is None or (op_type == 'Div' and k == 0):
                    raise _lib.UnsupportedInput(
                        f'vibecheck_nn_b200: {op_type} {name!r} without a constant factor')
                scale = np.asarray(c[k], np.float64)
                scale = 1.0 / scale if op_type == 'Div' else scale
                ops.append({'name': name, 'type': 'mul', 'inputs': [src(ins[1 - k])],
                            'scale': scale.reshape(-1)})
            else:
                raise _lib.UnsupportedInput(
                    f'vibecheck_nn_b200: ONNX op {op_type!r} at {name!r}')
            computed.add(name)
        refs = {}
        for op in ops:
            for i in op['inputs']:
                refs[i] = refs.get(i, 0) + 1
        return {'ops': ops, 'relu_names': relu_names,
                'fork_points': {n for n, k in refs.items() if k > 1},
                'n_relu': len(relu_names), 'input_name': self.input_name,
                'input_n': self.input_n, 'input_shape': self.input_shape}

    # -------------------------------------------------------------- replay
    def forward64(self, x):
        """Network output for input x (reshaped to the input shape), all in
        float64."""
        vals = {k: np.asarray(v, np.float64) if np.asarray(v).dtype.kind == 'f' else v
                for k, v in self.consts.items()}
        vals[self.input_name] = np.asarray(x, np.float64).reshape(self.input_shape)
        for op_type, ins, outs, attrs in self.nodes:
            if op_type == 'Constant':
                continue
            vals[outs[0]] = _eval(op_type, [vals.get(i) for i in ins], attrs)
        return np.asarray(vals[self.output_name], np.float64).reshape(-1)


def _eval(op_type, a, attrs):
    """One node on numpy arrays (float64 arithmetic for float inputs)."""
    if op_type in ('Identity', 'Dropout', 'Cast'):
        return a[0]
    if op_type == 'Add':
        return a[0] + a[1]
    if op_type == 'Sub':
        return a[0] - a[1]
    if op_type == 'Mul':
        return a[0] * a[1]
    if op_type == 'Div':
        return a[0] / a[1]
    if op_type == 'MatMul':
        return a[0] @ a[1]
    if op_type == 'Gemm':
        A = a[0].T if attrs.get('transA', 0) else a[0]
        B = a[1].T if attrs.get('transB', 0) else a[1]
        y = attrs.get('alpha', 1.0) * (A @ B)
        if len(a) > 2 and a[2] is not None:
            y = y + attrs.get('beta', 1.0) * a[2]
        return y
    if op_type == 'Relu':
        return np.maximum(a[0], 0.0)
    if op_type == 'Flatten':
        ax = attrs.get('axis', 1)
        sh = a[0].shape
        return a[0].reshape(int(np.prod(sh[:ax])), -1)
    if op_type == 'Reshape':
        shape = [int(s) for s in np.asarray(a[1]).reshape(-1)]
        shape = [a[0].shape[i] if s == 0 else s for i, s in enumerate(shape)]
        return a[0].reshape(shape)
    raise _lib.UnsupportedInput(f'vibecheck_nn_b200: ONNX op {op_type!r}')


def read_onnx(path_or_bytes):
    """Parse an ONNX model (a path, optionally .gz, or the file's bytes)."""
    if isinstance(path_or_bytes, (bytes, bytearray)):
        b = bytes(path_or_bytes)
    else:
        opener = gzip.open if str(path_or_bytes).endswith('.gz') else open
        with opener(path_or_bytes, 'rb') as f:
            b = f.read()
    graph = None
    for f, _, v in _fields(b):
        if f == 7:
            graph = v
    if graph is None:
        raise ValueError('ONNX model without a graph')
    nodes, consts, inputs, outputs = [], {}, [], []
    for f, _, v in _fields(graph):
        if f == 1:  # NodeProto
            ins, outs, op, attrs = [], [], '', {}
            for nf, _, nv in _fields(v):
                if nf == 1:
                    ins.append(nv.decode())
                elif nf == 2:
                    outs.append(nv.decode())
                elif nf == 4:
                    op = nv.decode()
                elif nf == 5:
                    k, val = _attribute(nv)
                    attrs[k] = val
            nodes.append((op, ins, outs, attrs))
            if op == 'Constant' and 'value' in attrs:
                consts[outs[0]] = attrs['value']
        elif f == 5:  # initializer
            name, arr = _tensor(v)
            consts[name] = arr
        elif f == 11:
            inputs.append(_value_info(v))
        elif f == 12:
            outputs.append(_value_info(v)[0])
    consts = {k: (np.asarray(v, np.float64) if np.asarray(v).dtype.kind == 'f' else np.asarray(v))
              for k, v in consts.items()}
    real_inputs = [(n, d) for n, d in inputs if n not in consts]
    if not real_inputs or not outputs:
        raise ValueError('ONNX graph without a data input or an output')
    return OnnxGraph(nodes, consts, real_inputs[0][0], real_inputs[0][1], outputs[0])
