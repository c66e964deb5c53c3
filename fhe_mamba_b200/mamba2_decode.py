"""Encrypted decode of a Mamba-2 chain payload from the command line, with the
flags of the reference's stage-1 decode binary that apply to this backend
(native/fideslib_stage0/src/stage1_mamba2_config.cpp:100-250, defaults from
stage1_mamba2_config.hpp:20-211):

    python -m fhe_mamba_b200.mamba2_decode --input-chain DIR --output-json PATH
        [--max-layers 0] [--tokens 4] [--ring-dim 131072]
        [--multiplicative-depth 44] [--scaling-mod-size 59] [--first-mod-size 60]
        [--num-large-digits 0] [--bootstrap-level-budget-cts 5]
        [--bootstrap-level-budget-stc 5] [--security 128-classic|not-set]
        [--secret-key-dist uniform-ternary|sparse-encapsulated]
        [--autoregressive-client-loop 0|1] [--tolerance 5e-2] [--refresh-passes 2]
        [--meta-bts 0|1] [--meta-bts-alpha 12] [--meta-bts-residual-layers 20,21]
        [--pt-cache-gib 5] [--seed 0]

Refreshes: by default every refresh is two-pass (the residual of the first
bootstrap, amplified by 2^12, bootstrapped again: the reference's Meta-BTS)
or one bootstrap with --refresh-passes 1; --meta-bts 0|1 selects the
reference decode's own policy instead (Meta-BTS only for carried values, the
gated norm's polynomial input, the residual at --meta-bts-residual-layers,
and the transient values of scheduled-normalization layers).

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
"""
from __future__ import annotations

import argparse
import json
import sys


def _bool(v: str) -> bool:
    if v in ("1", "true"):
        return True
    if v in ("0", "false"):
        return False
    raise argparse.ArgumentTypeError("expected 0, 1, false, or true")


def parse_args(argv=None):
    ap = argparse.ArgumentParser(prog="mamba2_decode", description=__doc__.split("\n\n")[0])
    ap.add_argument("--input-chain", required=True)
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
    ap.add_argument("--seed", type=int, default=0)
    return ap.parse_args(argv)


def run(args) -> dict:
    from .chain_payload import PayloadError, read_chain_payload, run_chain
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
    payload = read_chain_payload(args.input_chain, args.max_layers, args.autoregressive_client_loop)
    cc = CryptoContext(CCParams(ring_dim=args.ring_dim, multiplicative_depth=args.multiplicative_depth,
                                scaling_mod_size=args.scaling_mod_size, first_mod_size=args.first_mod_size,
                                num_large_digits=args.num_large_digits))
    cc.KeyGen(args.seed)
    cc.EvalBootstrapSetup((args.bootstrap_level_budget_cts, args.bootstrap_level_budget_stc),
                          sparse_hamming_weight=32 if args.secret_key_dist == "sparse-encapsulated" else 0)
    cc.EvalBootstrapKeyGen()
    result = run_chain(cc, payload, args.tokens, args.tolerance, args.autoregressive_client_loop,
                       passes=args.refresh_passes, cache_gb=args.pt_cache_gib, meta_bts=args.meta_bts,
                       meta_bts_residual_layers=residual_layers)
    result["parameters"].update({"multiplicative_depth": args.multiplicative_depth,
                                 "scaling_mod_size": args.scaling_mod_size, "first_mod_size": args.first_mod_size,
                                 "num_large_digits": args.num_large_digits, "security": args.security,
                                 "secret_key_dist": args.secret_key_dist,
                                 "bootstrap_level_budget": [args.bootstrap_level_budget_cts,
                                                            args.bootstrap_level_budget_stc],
                                 "max_layers": args.max_layers, "input_chain": str(args.input_chain)})
    if audit is not None:
        result["security_audit"] = audit
    return result


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
