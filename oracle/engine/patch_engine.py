"""Write the CUDA build of the reference engine's forward_v2.c: a copy of the
engine's own file with the two hook calls of rabbit_cuda_engine.c added (at the
top of moe_step and of rabbit_ref_v2_greedy) and that file appended.

    python3 patch_engine.py <engine src/forward_v2.c> <output .c>

The output goes to the build folder only (oracle/_ref); nothing of the engine's
source is kept in this repository. Anchors are the two functions' signature
lines; the script fails loudly if either is missing."""
import sys
from pathlib import Path

MOE = "static void moe_step(const RabbitModel *m, const RefV2Weights *w, int layer, float *h) {"
GREEDY = "int rabbit_ref_v2_greedy(RabbitModel *m, const char *prompt, int n_new,"

DECL_MOE = ("static int rabbit_cuda_hook_moe_step(const RabbitModel *m, const RefV2Weights *w, "
            "int layer, float *h);\n")
CALL_MOE = "    if (rabbit_cuda_hook_moe_step(m, w, layer, h)) return;\n"
DECL_GREEDY = ("static int rabbit_cuda_hook_greedy(RabbitModel *m, const char *prompt, int n_new, "
               "int *out_ids, int max_ids);\n")
CALL_GREEDY = ("    { const int rc_n = rabbit_cuda_hook_greedy(m, prompt, n_new, out_ids, max_ids);\n"
               "      if (rc_n != -2) return rc_n; }\n")


def patch(text: str) -> str:
    i = text.index(MOE)
    j = i + len(MOE)
    text = text[:i] + DECL_MOE + text[i:j] + "\n" + CALL_MOE + text[j + 1:]
    i = text.index(GREEDY)
    j = text.index("{", i) + 1  # the body's opening brace, after the parameter list
    text = text[:i] + DECL_GREEDY + text[i:j] + "\n" + CALL_GREEDY + text[j + 1:]
    return text + '\n#include "rabbit_cuda_engine.c"\n'


def main() -> int:
    src, out = Path(sys.argv[1]), Path(sys.argv[2])
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(patch(src.read_text()))
    return 0


if __name__ == "__main__":
    sys.exit(main())
