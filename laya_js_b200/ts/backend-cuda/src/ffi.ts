/**
 * Runtime-neutral binding of include/laya_cuda.h: koffi on Node, bun:ffi on
 * Bun, Deno.dlopen on Deno — the three routes the reference's native backend
 * already uses (packages/backend-mlx/src/ffi.ts:169-318).
 *
 * Conventions of the C ABI: every call returns int32 (0 = ok); the message of
 * a failure is read with lc_last_error(). Tensor handles are uint64 values
 * below 2^53 and cross as JS numbers. Out-parameters point into one
 * long-lived scratch buffer.
 */
import { createRequire } from "node:module";

const require = (id: string) => createRequire(import.meta.url)(id);

// h = handle (u64), p = pointer to a buffer, i = i32, d = f64, z = size_t
type A = "h" | "p" | "i" | "d" | "z";
const OP1: A[] = ["p", "h"];
const OP2: A[] = ["p", "h", "h"];
const RED: A[] = ["p", "h", "i", "i"];

export const SYMBOLS: Record<string, A[]> = {
  lc_init: ["i"], lc_destroy: [], lc_set_stream: ["h"], lc_supports: ["i", "p"], lc_stats: ["p", "p", "p"],
  lc_from_host: ["p", "i", "p", "i", "p", "z"], lc_read: ["h", "p", "z"], lc_tensor_free: ["h"],
  lc_tensor_info: ["h", "p", "p", "p"], lc_flush: [],
  lc_reshape: ["p", "h", "p", "i"], lc_transpose: ["p", "h", "p", "i"], lc_slice: ["p", "h", "p", "p", "i"],
  lc_split: ["p", "h", "i", "i"], lc_concat: ["p", "p", "i", "i"], lc_cast: ["p", "h", "i"],
  lc_add: OP2, lc_sub: OP2, lc_mul: OP2, lc_div: OP2, lc_maximum: OP2, lc_where: ["p", "h", "h", "h"],
  lc_scale: ["p", "h", "d"], lc_exp: OP1, lc_log: OP1, lc_relu: OP1, lc_gelu: OP1,
  lc_sum: RED, lc_max: RED, lc_softmax: ["p", "h", "i"], lc_sort: ["p", "h", "i"],
  lc_matmul: OP2, lc_linear: ["p", "h", "h", "h"], lc_layer_norm: ["p", "h", "h", "h", "d"],
  lc_embedding: OP2, lc_gather_rows: OP2, lc_rope: ["p", "h", "d"], lc_sdpa: ["p", "h", "h", "h", "h", "d"],
  lc_geglu: OP1, lc_mean_pool: OP2,
  lc_from_host_quantized: ["p", "p", "p", "h", "h", "i", "i", "i", "p", "i", "p", "p", "i"],
  lc_quantized_linear: ["p", "h", "h", "h", "h", "i", "i", "i", "h"],
  lc_quantized_embedding: ["p", "h", "h", "h", "i", "i", "i", "h"],
  lc_equal: OP2, lc_not_equal: OP2, lc_less: OP2, lc_less_equal: OP2, lc_greater: OP2, lc_greater_equal: OP2,
  lc_logical_and: OP2, lc_logical_or: OP2, lc_logical_not: OP1, lc_sqrt: OP1, lc_rsqrt: OP1, lc_pow: OP2,
  lc_neg: OP1, lc_abs: OP1, lc_tanh: OP1, lc_sigmoid: OP1, lc_erf: OP1,
  lc_argmax: RED, lc_argmin: RED, lc_mean: RED, lc_min: RED, lc_cumsum: ["p", "h", "i"],
  lc_graph_capture_begin: [], lc_graph_capture_end: ["p"], lc_graph_capture_abort: [], lc_graph_launch: ["h"],
  lc_graph_destroy: ["h"], lc_copy_into: ["h", "h"],
};

type Fn = (...a: unknown[]) => number;
export interface Native {
  call(name: string, ...args: unknown[]): void;
  lastError(): string;
  addressOf(a: ArrayBufferView): number;
  runtime: "node" | "bun" | "deno";
}

function wrap(fns: Record<string, Fn>, lastError: () => string, addressOf: (a: ArrayBufferView) => number, runtime: Native["runtime"]): Native {
  return {
    runtime,
    lastError,
    addressOf,
    call(name, ...args) {
      const f = fns[name];
      if (!f) throw new Error(`liblaya_cuda: unknown symbol ${name}`);
      if (f(...args) !== 0) throw new Error(lastError());
    },
  };
}

function openNode(path: string): Native {
  const koffi = require("koffi");
  const T: Record<A, string> = { h: "uint64_t", p: "void *", i: "int32_t", d: "double", z: "size_t" };
  const lib = koffi.load(path);
  const fns: Record<string, Fn> = {};
  for (const [k, args] of Object.entries(SYMBOLS)) fns[k] = lib.func(k, "int32_t", args.map((a) => T[a]));
  const err = lib.func("lc_last_error", "const char *", []);
  return wrap(fns, () => String(err()), (a) => Number(koffi.address(a)), "node");
}

function openBun(path: string): Native {
  const ffi = require("bun:ffi");
  const T: Record<A, string> = { h: "u64", p: "ptr", i: "i32", d: "f64", z: "usize" };
  const defs: Record<string, { args: string[]; returns: string }> = { lc_last_error: { args: [], returns: "cstring" } };
  for (const [k, args] of Object.entries(SYMBOLS)) defs[k] = { args: args.map((a) => T[a]), returns: "i32" };
  const lib = ffi.dlopen(path, defs);
  return wrap(lib.symbols as Record<string, Fn>, () => String(lib.symbols.lc_last_error()), (a) => Number(ffi.ptr(a)), "bun");
}

function openDeno(path: string): Native {
  const D = (globalThis as { Deno?: any }).Deno;
  const T: Record<A, string> = { h: "u64", p: "buffer", i: "i32", d: "f64", z: "usize" };
  const defs: Record<string, { parameters: string[]; result: string }> = { lc_last_error: { parameters: [], result: "pointer" } };
  for (const [k, args] of Object.entries(SYMBOLS)) defs[k] = { parameters: args.map((a) => T[a]), result: "i32" };
  const lib = D.dlopen(path, defs);
  const last = () => {
    const p = lib.symbols.lc_last_error();
    return p ? new D.UnsafePointerView(p).getCString() : "liblaya_cuda error";
  };
  return wrap(lib.symbols as Record<string, Fn>, last, (a) => Number(D.UnsafePointer.value(D.UnsafePointer.of(a))), "deno");
}

export function openNative(path: string): Native {
  const g = globalThis as { Bun?: unknown; Deno?: unknown };
  if (g.Bun) return openBun(path);
  if (g.Deno) return openDeno(path);
  return openNode(path);
}
