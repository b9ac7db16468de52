/**
 * @johnhenry/backend-cuda — the tensor-backend contract
 * (packages/tensor-backend/src/index.ts:139-317) on NVIDIA B200 through
 * liblaya_cuda.so (include/laya_cuda.h). One op = one C call, the way
 * @johnhenry/backend-mlx makes one mlx-c call per op.
 *
 *   import { createCudaBackend } from "@johnhenry/backend-cuda";
 *   const b = createCudaBackend({ device: 0 });
 */
import type { Backend, DType, HostQuantized, HostTensor, QuantizedLinearOptions, QuantizedTensor, Shape, Tensor } from "@johnhenry/tensor-backend";
import { allocHost, validateQuantized } from "@johnhenry/tensor-backend";
import { openNative, type Native } from "./ffi.ts";
import { resolveLib } from "./lib.ts";

export { resolveLib, cudaPlatformSupported } from "./lib.ts";

const DTYPES: DType[] = ["f32", "f16", "bf16", "i32", "bool", "u8", "i8", "u16", "i16", "u32", "u64", "i64", "f64"];
const CODE = new Map(DTYPES.map((d, i) => [d, i] as const));
const MODE = { symmetric: 0, affine: 1 } as const;

export class CudaTensor implements Tensor {
  disposed = false;
  constructor(readonly handle: number, readonly shape: Shape, readonly dtype: DType) {}
}

export interface CudaBackendOptions {
  device?: number;
  libPath?: string;
}

export function createCudaBackend(opts: CudaBackendOptions = {}): Backend<CudaTensor> & { stats(): Record<string, number> } {
  const N: Native = openNative(resolveLib(opts.libPath));
  N.call("lc_init", opts.device ?? 0);
  const out = new BigUint64Array(64);  // out-parameter scratch (handles)
  const i32 = new Int32Array(16);
  const i64 = new BigInt64Array(16);
  const scopes: CudaTensor[][] = [];
  const live = new FinalizationRegistry<number>((h) => {
    try {
      N.call("lc_tensor_free", h);
    } catch {
      /* already freed by destroy() */
    }
  });

  const wrap = (h: number): CudaTensor => {
    N.call("lc_tensor_info", h, i32.subarray(0, 1), i32.subarray(1, 2), i64.subarray(0, 8));
    const nd = i32[1]!;
    const t = new CudaTensor(h, Array.from(i64.subarray(0, nd), Number), DTYPES[i32[0]!]!);
    live.register(t, h, t);
    scopes[scopes.length - 1]?.push(t);
    return t;
  };
  const H = (t: CudaTensor | null | undefined, what: string): number => {
    if (!t) return 0;
    if (t.disposed) throw new Error(`${what}: tensor used after dispose`);
    return t.handle;
  };
  const op = (name: string, ...args: unknown[]): CudaTensor => {
    N.call(name, out, ...args);
    return wrap(Number(out[0]));
  };
  const shapeArg = (s: readonly number[]) => BigInt64Array.from(s.map((d) => BigInt(d)));
  const un = (name: string) => (x: CudaTensor) => op(name, H(x, name));
  const bin = (name: string) => (a: CudaTensor, b: CudaTensor) => op(name, H(a, name), H(b, name));
  const red = (name: string) => (x: CudaTensor, axis: number, keepDims = false) => op(name, H(x, name), axis, keepDims ? 1 : 0);

  const b = {
    name: "cuda",
    supports: (d: DType) => CODE.has(d),
    async fromHost(t: HostTensor): Promise<CudaTensor> {
      const code = CODE.get(t.dtype);
      if (code === undefined) throw new TypeError(`fromHost: unknown dtype ${t.dtype}`);
      const data = t.data as ArrayBufferView;
      return op("lc_from_host", code, shapeArg(t.shape), t.shape.length, data, data.byteLength);
    },
    async read(t: CudaTensor): Promise<HostTensor> {
      const n = t.shape.reduce((a, d) => a * d, 1);
      const data = allocHost(t.dtype, n);
      N.call("lc_read", H(t, "read"), data, (data as ArrayBufferView).byteLength);
      return { dtype: t.dtype, shape: [...t.shape], data };
    },
    dispose(t: CudaTensor) {
      if (!t || t.disposed) return;
      t.disposed = true;
      live.unregister(t);
      N.call("lc_tensor_free", t.handle);
    },
    scope<R>(fn: () => R): R {
      const frame: CudaTensor[] = [];
      scopes.push(frame);
      let r: R;
      try {
        r = fn();
      } catch (e) {
        scopes.pop();
        for (const t of frame) b.dispose(t);
        throw e;
      }
      scopes.pop();
      const keep = new Set<CudaTensor>();
      if (r instanceof CudaTensor) {
        keep.add(r);
      } else if (Array.isArray(r)) {
        for (const x of r) if (x instanceof CudaTensor) keep.add(x);
      } else if (r && typeof r === "object") {
        for (const x of Object.values(r)) if (x instanceof CudaTensor) keep.add(x);
      }
      for (const t of frame) {
        if (keep.has(t)) scopes[scopes.length - 1]?.push(t);
        else b.dispose(t);
      }
      return r;
    },
    flush: () => N.call("lc_flush"),
    destroy: () => N.call("lc_destroy"),
    stats() {
      const s = new BigInt64Array(3);
      N.call("lc_stats", s.subarray(0, 1), s.subarray(1, 2), s.subarray(2, 3));
      return { liveTensors: Number(s[0]), liveBytes: Number(s[1]), launches: Number(s[2]) };
    },

    reshape: (x: CudaTensor, s: Shape) => op("lc_reshape", H(x, "reshape"), shapeArg(s), s.length),
    transpose: (x: CudaTensor, perm: readonly number[]) => op("lc_transpose", H(x, "transpose"), Int32Array.from(perm), perm.length),
    slice: (x: CudaTensor, begin: readonly number[], end: readonly number[]) =>
      op("lc_slice", H(x, "slice"), shapeArg(begin), shapeArg(end), begin.length),
    split(x: CudaTensor, parts: number, axis: number): CudaTensor[] {
      const outs = new BigUint64Array(parts);
      N.call("lc_split", outs, H(x, "split"), parts, axis);
      return Array.from(outs, (h) => wrap(Number(h)));
    },
    concat: (xs: readonly CudaTensor[], axis: number) => op("lc_concat", BigUint64Array.from(xs.map((x) => BigInt(H(x, "concat")))), xs.length, axis),
    cast: (x: CudaTensor, d: DType) => op("lc_cast", H(x, "cast"), CODE.get(d)!),

    add: bin("lc_add"), sub: bin("lc_sub"), mul: bin("lc_mul"), div: bin("lc_div"), maximum: bin("lc_maximum"),
    where: (c: CudaTensor, x: CudaTensor, y: CudaTensor) => op("lc_where", H(c, "where"), H(x, "where"), H(y, "where")),
    scale: (x: CudaTensor, s: number) => op("lc_scale", H(x, "scale"), s),
    exp: un("lc_exp"), log: un("lc_log"), relu: un("lc_relu"), gelu: un("lc_gelu"),
    sum: red("lc_sum"), max: red("lc_max"),
    softmax: (x: CudaTensor, axis: number) => op("lc_softmax", H(x, "softmax"), axis),
    sort: (x: CudaTensor, axis: number) => op("lc_sort", H(x, "sort"), axis),
    matmul: bin("lc_matmul"),
    linear: (x: CudaTensor, w: CudaTensor, bias?: CudaTensor | null) => op("lc_linear", H(x, "linear"), H(w, "linear"), H(bias, "linear")),
    layerNorm: (x: CudaTensor, w: CudaTensor | null, bias: CudaTensor | null, eps: number) =>
      op("lc_layer_norm", H(x, "layerNorm"), H(w, "layerNorm"), H(bias, "layerNorm"), eps),
    embedding: bin("lc_embedding"),
    gatherRows: bin("lc_gather_rows"),
    rope: (x: CudaTensor, base: number) => op("lc_rope", H(x, "rope"), base),
    sdpa: (q: CudaTensor, k: CudaTensor, v: CudaTensor, m: CudaTensor | null, s: number) =>
      op("lc_sdpa", H(q, "sdpa"), H(k, "sdpa"), H(v, "sdpa"), H(m, "sdpa"), s),
    geglu: un("lc_geglu"),
    meanPool: bin("lc_mean_pool"),

    async fromHostQuantized(h: HostQuantized, dtype: DType): Promise<QuantizedTensor<CudaTensor> | null> {
      validateQuantized(h);
      if (dtype !== "f32" && dtype !== "f16" && dtype !== "bf16") return null;
      const [n, k] = h.shape;
      const o = new BigUint64Array(3);
      N.call("lc_from_host_quantized", o.subarray(0, 1), o.subarray(1, 2), o.subarray(2, 3), n, k, h.bits, h.groupSize, MODE[h.mode], h.data,
        CODE.get(h.scales.dtype)!, h.scales.data, h.biases ? h.biases.data : null, CODE.get(dtype)!);
      return { shape: [n, k], bits: h.bits, groupSize: h.groupSize, mode: h.mode, dtype, native: true,
        w: wrap(Number(o[0])), scales: wrap(Number(o[1])), biases: o[2] ? wrap(Number(o[2])) : null };
    },
    quantizedLinear: (x: CudaTensor, w: CudaTensor, s: CudaTensor, bi: CudaTensor | null, q: QuantizedLinearOptions, bias?: CudaTensor | null) =>
      op("lc_quantized_linear", H(x, "quantizedLinear"), H(w, "quantizedLinear"), H(s, "quantizedLinear"), H(bi, "quantizedLinear"), q.bits,
        q.groupSize, MODE[q.mode], H(bias, "quantizedLinear")),
    quantizedEmbedding: (w: CudaTensor, s: CudaTensor, bi: CudaTensor | null, q: QuantizedLinearOptions, ids: CudaTensor) =>
      op("lc_quantized_embedding", H(w, "quantizedEmbedding"), H(s, "quantizedEmbedding"), H(bi, "quantizedEmbedding"), q.bits, q.groupSize,
        MODE[q.mode], H(ids, "quantizedEmbedding")),

    equal: bin("lc_equal"), notEqual: bin("lc_not_equal"), less: bin("lc_less"), lessEqual: bin("lc_less_equal"),
    greater: bin("lc_greater"), greaterEqual: bin("lc_greater_equal"), logicalAnd: bin("lc_logical_and"), logicalOr: bin("lc_logical_or"),
    logicalNot: un("lc_logical_not"), sqrt: un("lc_sqrt"), rsqrt: un("lc_rsqrt"), pow: bin("lc_pow"), neg: un("lc_neg"), abs: un("lc_abs"),
    tanh: un("lc_tanh"), sigmoid: un("lc_sigmoid"), erf: un("lc_erf"),
    argmax: red("lc_argmax"), argmin: red("lc_argmin"), mean: red("lc_mean"), min: red("lc_min"),
    cumsum: (x: CudaTensor, axis: number) => op("lc_cumsum", H(x, "cumsum"), axis),

    /**
     * index.ts:244-245. CUDA-graph capture per input signature (dtypes and
     * shapes): the first call of a signature runs `fn` eagerly, then records
     * it on graph-owned input tensors; later calls copy their arguments in,
     * replay the graph (one launch) and return copies of its outputs. `fn`
     * must be pure in its tensor arguments (captured tensors are constants,
     * as under backend-mlx's compile).
     */
    compile<A extends CudaTensor[], R>(fn: (...args: A) => R): (...args: A) => R {
      type Rec = { graph: number; ins: CudaTensor[]; outs: CudaTensor[]; rebuild: (xs: CudaTensor[]) => R };
      const recs = new Map<string, Rec>();
      const flatten = (r: unknown): { flat: CudaTensor[]; rebuild: (xs: CudaTensor[]) => R } => {
        if (r instanceof CudaTensor) return { flat: [r], rebuild: (xs) => xs[0] as R };
        if (Array.isArray(r)) return { flat: r as CudaTensor[], rebuild: (xs) => xs as R };
        if (r && typeof r === "object") {
          const keys = Object.keys(r);
          return { flat: keys.map((k) => (r as Record<string, CudaTensor>)[k]!), rebuild: (xs) => Object.fromEntries(keys.map((k, i) => [k, xs[i]])) as R };
        }
        throw new TypeError("compile: outputs must be a tensor, an array or an object of tensors");
      };
      const zeros = (t: CudaTensor) => {
        const n = t.shape.reduce((a, d) => a * d, 1);
        const data = allocHost(t.dtype, n) as ArrayBufferView;
        return op("lc_from_host", CODE.get(t.dtype)!, shapeArg(t.shape), t.shape.length, data, data.byteLength);
      };
      const record = (args: A, result: R): Rec => {
        const { flat, rebuild } = flatten(result);
        const saved = scopes.splice(0, scopes.length);  // graph tensors belong to no caller scope
        try {
          const ins = args.map(zeros);
          const outs = flat.map(zeros);
          N.call("lc_graph_capture_begin");
          try {
            b.scope(() => {
              const views = ins.map((t) => b.reshape(t, t.shape)) as unknown as A;
              const got = flatten(fn(...views)).flat;
              got.forEach((t, i) => N.call("lc_copy_into", outs[i]!.handle, H(t, "compile")));
              return null;
            });
            N.call("lc_graph_capture_end", out);
          } catch (e) {
            N.call("lc_graph_capture_abort");
            for (const t of [...ins, ...outs]) b.dispose(t);
            throw e;
          }
          return { graph: Number(out[0]), ins, outs, rebuild };
        } finally {
          scopes.push(...saved);
        }
      };
      return (...args: A): R => {
        const sig = args.map((t) => `${t.dtype}[${t.shape.join(",")}]`).join(";");
        const rec = recs.get(sig);
        if (!rec) {
          const result = fn(...args);
          recs.set(sig, record(args, result));
          return result;
        }
        rec.ins.forEach((slot, i) => N.call("lc_copy_into", slot.handle, H(args[i], "compiled call")));
        N.call("lc_graph_launch", rec.graph);
        return rec.rebuild(rec.outs.map((o) => b.cast(o, o.dtype)));
      };
    },
  };
  return b as unknown as Backend<CudaTensor> & { stats(): Record<string, number> };
}
