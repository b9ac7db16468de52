/**
 * Locates liblaya_cuda.so. Same rule as the MLX backend's library resolution
 * (packages/backend-mlx/src/lib.ts:473-511): an explicit path or
 * $LAYA_CUDA_LIB wins, and when it is set but missing that is an error,
 * never a silent fallback; otherwise the copy bundled next to this package.
 */
import { existsSync } from "node:fs";
import { fileURLToPath } from "node:url";

export function resolveLib(explicit?: string): string {
  const env = (globalThis as { process?: { env: Record<string, string | undefined> } }).process?.env?.LAYA_CUDA_LIB;
  const wanted = explicit ?? env;
  if (wanted) {
    if (!existsSync(wanted)) throw new Error(`liblaya_cuda: ${wanted} does not exist (LAYA_CUDA_LIB / libPath set but missing)`);
    return wanted;
  }
  const bundled = fileURLToPath(new URL("../native/liblaya_cuda.so", import.meta.url));
  if (!existsSync(bundled)) throw new Error(`liblaya_cuda: not built; run \`python -m laya_js_b200.build\` and copy liblaya_cuda.so to ${bundled}`);
  return bundled;
}

export function cudaPlatformSupported(): boolean {
  const p = (globalThis as { process?: { platform: string; arch: string } }).process;
  return !!p && p.platform === "linux" && p.arch === "x64";
}
