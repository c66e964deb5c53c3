"""Encrypted decode of a Mamba-2 chain payload from the command line, with the
flags of the reference's stage-1 decode binary that apply to this backend
(native/fideslib_stage0/src/stage1_mamba2_config.cpp:100-250, defaults from
stage1_mamba2_config.hpp:20-211):

    python -m fhe_mamba_b200.mamba2_decode (--input-chain DIR | --input LAYER_DIR) --output-json PATH
        [--max-layers 0] [--tokens 4] [--ring-dim 131072]
        [--multiplicative-depth 44] [--scaling-mod-size 59] [--first-mod-size 60]
        [--num-large-digits 0] [--bootstrap-level-budget-cts 5]
        [--bootstrap-level-budget-stc 5] [--security 128-classic|not-set]
        [--secret-key-dist uniform-ternary|sparse-encapsulated]
        [--autoregressive-client-loop 0|1] [--tolerance 5e-2] [--refresh-passes 2]
        [--meta-bts 0|1] [--meta-bts-alpha 12] [--meta-bts-residual-layers 20,21]
        [--pt-cache-gib 5] [--seed S] [--debug-layer-errors 0|1]
        [--rotation-keys full|compact|balanced] [--rotation-key-gib 45]
        [--process-role inline|client-init|server-eval|client-decrypt --handoff-dir DIR]

Refreshes: by default every refresh is two-pass (the residual of the first
bootstrap, amplified by 2^12, bootstrapped again: the reference's Meta-BTS)
or one bootstrap with --refresh-passes 1; --meta-bts 0|1 selects the
reference decode's own policy instead (Meta-BTS only for carried values, the
gated norm's polynomial input, the residual at --meta-bts-residual-layers,
and the transient values of scheduled-normalization layers).

Process separation (--process-role, the reference's handoff protocol):
client-init keeps the secret key in DIR/client, writes the evaluation keys to
DIR/server and the encrypted test inputs to DIR/exchange; server-eval loads
only DIR/server, evaluates and writes DIR/exchange/output_t*.ct; client-decrypt
decrypts them and checks them against the payload's reference.  Each role is
its own process with the same parameter flags.

The result document goes to --output-json; the exit code is 0 when the
decrypted outputs are within --tolerance of the payload's polynomial-circuit
reference (and, with the client loop, the greedy ids match), 1 when not, 2 on
an error (whose message is also written to --output-json).  --security
128-classic refuses parameters above the classical-128 bound of the
homomorphic encryption standard (the audit of ``security_audit``), as the
reference's SetSecurityLevel(HEStd_128_classic) does; --num-large-digits 0
picks the fewest key-switching digits (at least 3) that pass it (4 at the
default ring 2^17, depth 44: 45 Q primes, 12 P primes, 3376 of 3523 bits),
or 3 with --security not-set.  The main secret is
uniform ternary; ``sparse-encapsulated`` switches bootstrapping to a sparse
secret of Hamming weight 32 (the reference's SPARSE_ENCAPSULATED); a sparse
main secret (``sparse-ternary``, the reference's default) is not supported.
Keys derive from --seed (reproducible runs); without it the seed is drawn
from the operating system, and it is never written to the result.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np


def _bool(v: str) -> bool:
    if v in ("1", "true"):
        return True
    if v in ("0", "false"):
        return False
    raise argparse.ArgumentTypeError("expected 0, 1, false, or true")


def parse_args(argv=None):
    ap = argparse.ArgumentParser(prog="mamba2_decode", description=__doc__.split("\n\n")[0])
    src = ap.add_mutually_exclusive_group(required=True)
    src.add_argument("--input-chain")
    src.add_argument("--input")
    ap.add_argument("--output-json", required=True)
    ap.add_argument("--max-layers", type=int, default=0)
    ap.add_argument("--tokens", type=int, default=4)
    ap.add_argument("--ring-dim", type=int, default=131072)
    ap.add_argument("--multiplicative-depth", type=int, default=44)
    ap.add_argument("--scaling-mod-size", type=int, default=59)
    ap.add_argument("--first-mod-size", type=int, default=60)
    ap.add_argument("--num-large-digits", type=int, default=0)
    ap.add_argument("--bootstrap-level-budget-cts", type=int, default=5)
    ap.add_argument("--bootstrap-level-budget-stc", type=int, default=5)
    ap.add_argument("--security", choices=("128-classic", "not-set"), default="128-classic")
    ap.add_argument("--secret-key-dist", default="uniform-ternary")
    ap.add_argument("--autoregressive-client-loop", type=_bool, default=False)
    ap.add_argument("--tolerance", type=float, default=5e-2)
    ap.add_argument("--refresh-passes", type=int, choices=(1, 2), default=2)
    ap.add_argument("--meta-bts", type=_bool, default=None)
    ap.add_argument("--meta-bts-alpha", type=int, default=12)
    ap.add_argument("--state-meta-bts-alpha", type=int, default=-1)
    ap.add_argument("--meta-bts-residual-layers", default="")
    ap.add_argument("--pt-cache-gib", type=float, default=5.0)
    ap.add_argument("--seed", type=int, default=None)
    ap.add_argument("--debug-layer-errors", type=_bool, default=False)
    ap.add_argument("--rotation-keys", choices=("full", "compact", "balanced"), default="full")
    ap.add_argument("--rotation-key-gib", type=float, default=45.0)
    ap.add_argument("--process-role", choices=ROLES, default="inline")
    ap.add_argument("--handoff-dir", default="")
    return ap.parse_args(argv)


ROLES = ("inline", "client-init", "server-eval", "client-decrypt")


def handoff_paths(root):
    """client/ (the secret), server/ (evaluation keys only), exchange/
    (ciphertexts), as the reference's handoff_paths
    (native/fideslib_stage0/src/stage1_mamba2_process.cpp:28-35)."""
    root = Path(root)
    return {"root": root, "client": root / "client", "server": root / "server", "exchange": root / "exchange"}


def server_secret_files(paths) -> int:
    """Files under server/ that could hold a secret (the server must have none)."""
    if not paths["server"].is_dir():
        return 0
    return sum(1 for f in paths["server"].iterdir() if "secret" in f.name or f.name == CLIENT_KEYS)


CLIENT_KEYS = "client.keys"   # public, evaluation and secret key (client/)
SERVER_KEYS = "eval.keys"     # public and evaluation keys (server/)


def run(args, context_factory=None) -> dict:
    """One invocation; `context_factory` makes the CryptoContext (default: the
    device library with the command line's parameters)."""
    from .chain_payload import PayloadError, read_chain_payload, read_layer_as_chain, run_chain
    from .ckks import CCParams, CryptoContext
    from .program import security_audit

    if args.meta_bts_alpha != 12 or args.state_meta_bts_alpha not in (-1, 12):
        raise PayloadError("the refresh amplifies the Meta-BTS residual by 2^12 (--meta-bts-alpha 12)")
    try:
        residual_layers = {int(t) for t in args.meta_bts_residual_layers.split(",") if t}
    except ValueError as e:
        raise PayloadError("--meta-bts-residual-layers expects comma-separated layer indices") from e
    if args.secret_key_dist not in ("uniform-ternary", "sparse-encapsulated"):
        raise PayloadError(f"unsupported --secret-key-dist {args.secret_key_dist} "
                           "(uniform-ternary or sparse-encapsulated)")
    log_n = int(args.ring_dim).bit_length() - 1
    audit = None
    if args.security == "128-classic":
        def check(dnum):
            return security_audit(log_n, args.multiplicative_depth, args.scaling_mod_size, args.first_mod_size,
                                  dnum)
        if args.num_large_digits == 0:
            for dnum in range(3, 16):
                audit = check(dnum)
                if audit.get("passed"):
                    args.num_large_digits = dnum
                    break
        else:
            audit = check(args.num_large_digits)
        if not audit.get("passed"):
            raise PayloadError("parameters exceed the classical-128 bound: " + json.dumps(audit))
    elif args.num_large_digits == 0:
        args.num_large_digits = 3
    if args.input_chain:
        payload = read_chain_payload(args.input_chain, args.max_layers, args.autoregressive_client_loop)
    else:
        if args.autoregressive_client_loop:
            raise PayloadError("autoregressive-client-loop needs --input-chain")
        payload = read_layer_as_chain(args.input)
    if args.process_role != "inline":
        if not args.handoff_dir:
            raise PayloadError(f"--process-role {args.process_role} needs --handoff-dir")
        if args.autoregressive_client_loop:
            raise PayloadError("the autoregressive client loop runs inline only")
        if args.secret_key_dist == "sparse-encapsulated":
            raise PayloadError("sparse-secret bootstrapping keys are not serialized; use uniform-ternary")
        if args.tokens < 1 or args.tokens > payload.n_test_tokens:
            raise PayloadError("--tokens exceeds n_test_tokens in the chain payload")
    factory = context_factory or (lambda: CryptoContext(CCParams(
        ring_dim=args.ring_dim, multiplicative_depth=args.multiplicative_depth,
        scaling_mod_size=args.scaling_mod_size, first_mod_size=args.first_mod_size,
        num_large_digits=args.num_large_digits)))
    if args.seed is None:  # keys derive from the seed: without one, draw it from the OS
        import secrets
        args.seed = secrets.randbits(63) | 1
    budget = (args.bootstrap_level_budget_cts, args.bootstrap_level_budget_stc)
    if args.rotation_key_gib <= 0:
        raise PayloadError("--rotation-key-gib must be positive")
    chain_options = dict(passes=args.refresh_passes, cache_gb=args.pt_cache_gib, meta_bts=args.meta_bts,
                         meta_bts_residual_layers=residual_layers, rotation_keys=args.rotation_keys,
                         rotation_key_gib=args.rotation_key_gib)
    if args.process_role == "inline":
        cc = factory()
        cc.KeyGen(args.seed)
        cc.EvalBootstrapSetup(budget, sparse_hamming_weight=32 if args.secret_key_dist == "sparse-encapsulated"
                              else 0)
        cc.EvalBootstrapKeyGen()
        result = run_chain(cc, payload, args.tokens, args.tolerance, args.autoregressive_client_loop,
                           debug_layer_errors=args.debug_layer_errors, **chain_options)
    else:
        result = run_role(args, payload, factory, budget, chain_options)
    result["parameters"].update({"multiplicative_depth": args.multiplicative_depth,
                                 "scaling_mod_size": args.scaling_mod_size, "first_mod_size": args.first_mod_size,
                                 "num_large_digits": args.num_large_digits, "security": args.security,
                                 "secret_key_dist": args.secret_key_dist,
                                 "bootstrap_level_budget": [args.bootstrap_level_budget_cts,
                                                            args.bootstrap_level_budget_stc],
                                 "max_layers": args.max_layers, "input_chain": args.input_chain,
                                 "input": args.input,
                                 "process_role": args.process_role})
    if audit is not None:
        result["security_audit"] = audit
    return result


def run_role(args, payload, factory, budget, chain_options) -> dict:
    """The process-separated protocol of the reference's decode
    (stage1_mamba2_decode_fideslib.cpp:879-977, 1248-1275, 1446-1520,
    4646-4700): client-init makes the keys, keeps the secret in client/,
    puts the evaluation keys in server/ and the encrypted test inputs in
    exchange/; server-eval loads only server/ (it cannot decrypt or make
    keys), runs the layers and writes the encrypted outputs; client-decrypt
    loads client/ and checks the outputs against the payload's reference."""
    import os
    import time

    from .chain_payload import EncryptedChain, PayloadError

    paths = handoff_paths(args.handoff_dir)
    ex = paths["exchange"]
    role = args.process_role
    params = {"process_role": role, "tokens": args.tokens, "layers": len(payload.layers)}
    scope = {"client_server_process_separation": True, "server_secret_key_loaded": False}
    if role == "client-init":
        root = paths["root"]
        if root.exists() and (not root.is_dir() or any(root.iterdir())):
            raise PayloadError(f"refusing to reuse non-empty handoff root: {root}")
        for k in ("client", "server", "exchange"):
            paths[k].mkdir(parents=True, exist_ok=True)
        for k in ("root", "client", "server", "exchange"):
            os.chmod(paths[k], 0o700)
        cc = factory()
        cc.KeyGen(args.seed)
        cc.EvalBootstrapSetup(budget)
        cc.EvalBootstrapKeyGen()
        chain = EncryptedChain(cc, payload, **chain_options)
        cc.EvalRotateKeyGen(chain.rotation_steps())
        cc.SerializeKeys(paths["server"] / SERVER_KEYS)
        cc.SerializeKeys(paths["client"] / CLIENT_KEYS, include_secret=True)
        os.chmod(paths["client"] / CLIENT_KEYS, 0o600)
        for t in range(args.tokens):
            cc.SerializeCiphertext(chain.encrypt(payload.input_embeddings[t]), ex / f"input_t{t}.ct")
        return {"status": "passed", "passed": True, "parameters": params,
                "measurements": {"encrypted_inputs_written": args.tokens},
                "measurement_scope": dict(scope, full_model_correctness_claimed=False)}
    if role == "server-eval":
        if server_secret_files(paths):
            raise PayloadError("the server directory holds secret-key files")
        cc = factory()
        cc.DeserializeKeys(paths["server"] / SERVER_KEYS)
        cc.EvalBootstrapSetup(budget)
        cc.EvalBootstrapKeyGen()  # every key is in the bundle: nothing is generated
        chain = EncryptedChain(cc, payload, **chain_options)
        steps = []
        for t in range(args.tokens):
            ct = cc.DeserializeCiphertext(ex / f"input_t{t}.ct")
            t0 = time.perf_counter()
            out = chain.step_ct(ct)
            steps.append(time.perf_counter() - t0)
            cc.SerializeCiphertext(out, ex / f"output_t{t}.ct")
        return {"status": "passed", "passed": True, "parameters": params,
                "measurements": {"encrypted_outputs_written": args.tokens, "server_secret_key_files": 0,
                                 "eval_seconds": sum(steps), "token_step_seconds": steps,
                                 "refreshes": chain.refreshes(), "meta_bts_applied": chain.two_pass_refreshes()},
                "measurement_scope": dict(scope, encrypted_full_layer_chain_evaluated=payload.full_chain,
                                          full_model_correctness_claimed=False)}
    # client-decrypt
    cc = factory()
    cc.DeserializeKeys(paths["client"] / CLIENT_KEYS)
    last = payload.layers[-1].tensors
    exact = payload.expected_final if payload.full_chain else last["test_layer_output"]
    poly = payload.expected_poly_final if payload.full_chain else last.get("test_layer_output_poly")
    reference = poly if poly is not None else exact
    errors, ok = [], []
    for t in range(args.tokens):
        try:
            got = cc.Decrypt(cc.DeserializeCiphertext(ex / f"output_t{t}.ct")).GetRealPackedValue()
            got = np.asarray(got[:payload.d_model])
            err = float(np.max(np.abs(got - reference[t])))
            errors.append(err if np.isfinite(err) else float("inf"))
            ok.append(1)
        except Exception:  # a missing or corrupt output fails its token, as in the reference
            errors.append(float("inf"))
            ok.append(0)
    secret_files = server_secret_files(paths)
    max_error = max(errors)
    passed = max_error <= args.tolerance and secret_files == 0
    return {"status": "passed" if passed else "failed", "passed": passed,
            "parameters": dict(params, tolerance=args.tolerance),
            "measurements": {"correctness_reference": "polynomial-circuit" if poly is not None else "exact-legacy",
                             "max_abs_error": max_error, "per_token_max_abs_error": errors,
                             "per_token_decrypt_ok": ok, "server_secret_key_files": secret_files},
            "measurement_scope": dict(scope, full_model_correctness_claimed=payload.full_chain)}


def main(argv=None) -> int:
    args = parse_args(argv)
    try:
        result = run(args)
        code = 0 if result["passed"] else 1
    except Exception as e:  # the reference reports every failure in its artifact and exits 2
        result = {"schema": "fhemamba-stage1-mamba2-result-v1", "backend": "fhe_b200", "status": "error",
                  "passed": False, "error": f"{type(e).__name__}: {e}"}
        code = 2
    with open(args.output_json, "w") as f:
        json.dump(result, f, indent=1)
    print(json.dumps({k: result.get(k) for k in ("status", "passed", "error") if k in result}))
    return code


if __name__ == "__main__":
    sys.exit(main())
