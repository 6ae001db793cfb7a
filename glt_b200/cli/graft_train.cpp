// graft_train: the reference's grafting command line (grafting.hip:274-1290)
// driven entirely through the C ABI of libglt_b200 (include/glt_graft.h).
//
// Three modes, as in the reference:
//   training     --safetensors --domain-data --ood-data ... --output
//   --eval-only  --safetensors --eval-data [--checkpoint]
//   --shadow-eval --safetensors --eval-data [--checkpoint]
// Every reference flag is accepted with the reference's default and
// validation; unknown flags are ignored, as the reference's flag loop does.
// New flags: --graft-layout overlay|concat (overlay, the reference geometry,
// is the default; concat is the [base | graft] layout of the benchmarks).
// Outputs follow the reference: <output>_log.csv with one row per step, the
// key=value summary lines on stdout, the GRFT v4 checkpoint at --output, and
// <output>.graft_gemm_stats.json with --profile-graft-gemms.
#include <sys/stat.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

#include "glt_graft.h"

namespace {

struct GltFailure : std::runtime_error {
  using std::runtime_error::runtime_error;
};

#define CHECK(call)                                                                            \
  do {                                                                                         \
    const int _s = (call);                                                                     \
    if (_s != GLT_OK)                                                                          \
      throw GltFailure(std::string(#call) + " failed at " + __FILE__ + ":" +                   \
                       std::to_string(__LINE__) + ": " + glt_last_error());                    \
  } while (0)

const char* const kProfNames[] = {
    "gate_up_fwd", "down_fwd",  "delta_down", "qkv",     "o_proj",  "attn_fwd",   "dh",
    "recompute_swiglu_bwd", "wgrad_down", "wgrad_gate_up", "dx_gate_up", "do", "attn_bwd",
    "dx_qkv", "lm_head", "lm_dx", "cross_entropy", "delta_expand", "graft_dgrad", "rmsnorm",
    "rope", "adamw"};
static_assert(sizeof(kProfNames) / sizeof(kProfNames[0]) == GLT_PROF_KINDS,
              "one name per GLT_PROF_* kind");

void print_usage(const char* argv0) {
  std::cout
      << "Usage: " << argv0 << " --safetensors PATH --domain-data FILE.bin --ood-data FILE.bin [FILE.bin ...]\n"
      << "       --output CKPT [options]\n"
      << "   or: " << argv0 << " --eval-only|--shadow-eval --safetensors PATH --eval-data FILE.bin [--checkpoint CKPT]\n"
      << "Options (reference defaults): --domain-id 0 --max-domains 4 --steps 200 --lr 2e-4\n"
      << "  --batch-size 16 --max-len 512 --seed 42 --lm-loss-scale 1 --lambda-silence 5\n"
      << "  --checkpoint CKPT --session-id ID --init-deltas RAW.f32\n"
      << "  --hidden-dim 2048 --intermediate-dim 11008 --slice-dim 2752 --vocab-size 128256\n"
      << "  --num-layers 36 --num-heads 16 --num-kv-heads 4 --head-dim 0 --rope-theta 5e6\n"
      << "  --no-rope-layers 1,1,0,...  --beta1 0.9 --beta2 0.999 --adam-eps 1e-8\n"
      << "  --weight-decay 0.01 --grad-clip 1.0 --warmup-steps 20 --threads 256\n"
      << "  --graft-layer-start 0 --graft-layer-end 35 --graft-proj-gate 0 --graft-proj-up 0\n"
      << "  --graft-proj-down 1 --allow-expansion-trap --graft-gemm-backend rocblas|hipblaslt-selective\n"
      << "  --delta-bf16-mirror --use-aten-delta-input-grad --profile-graft-gemms\n"
      << "  --parity-dump DIR --parity-dump-layer N --contract-probe --verbose --help\n"
      << "  --graft-layout overlay|concat   (new; overlay is the reference geometry)\n"
      << "  --save-state STATE --resume-state STATE --stop-after K\n"
      << "      (new: fp32 graft + Adam moments + next step; --steps stays the schedule length,\n"
      << "       --stop-after ends this run after step K-1 of it)\n";
}

bool is_dir(const std::string& p) {
  struct stat sb;
  return stat(p.c_str(), &sb) == 0 && S_ISDIR(sb.st_mode);
}
bool exists(const std::string& p) {
  struct stat sb;
  return stat(p.c_str(), &sb) == 0;
}
long long file_size(const std::string& p) {
  struct stat s;
  return stat(p.c_str(), &s) == 0 ? static_cast<long long>(s.st_size) : -1;
}

std::string parent_of(const std::string& p) {
  const size_t k = p.find_last_of('/');
  return k == std::string::npos ? std::string() : p.substr(0, k);
}
// fs::path::replace_extension
std::string replace_ext(const std::string& p, const std::string& ext) {
  const size_t slash = p.find_last_of('/');
  const size_t dot = p.find_last_of('.');
  if (dot != std::string::npos && (slash == std::string::npos || dot > slash) && dot != slash + 1)
    return p.substr(0, dot) + ext;
  return p + ext;
}

struct Tokens {
  int32_t num_sequences = 0, seq_len = 0;
  std::vector<int32_t> tokens;
};

bool load_bin(const std::string& path, Tokens* t) {
  if (glt_load_bin(path.c_str(), &t->num_sequences, &t->seq_len, nullptr, 0) != GLT_OK) {
    std::cerr << "Error: " << glt_last_error() << "\n";
    return false;
  }
  t->tokens.resize(static_cast<size_t>(t->num_sequences) * t->seq_len);
  if (glt_load_bin(path.c_str(), &t->num_sequences, &t->seq_len, t->tokens.data(),
                   static_cast<int64_t>(t->tokens.size())) != GLT_OK) {
    std::cerr << "Error: " << glt_last_error() << "\n";
    return false;
  }
  return true;
}

void write_raw(const std::string& path, const void* data, size_t bytes) {
  std::ofstream f(path, std::ios::binary);
  f.write(static_cast<const char*>(data), static_cast<std::streamsize>(bytes));
}

int64_t used_mb() {
  int64_t used = 0, total = 0;
  if (glt_device_memory(&used, &total) != GLT_OK) return 0;
  return used / 1024 / 1024;
}

// Creates the model and loads the base weights; lm_head tying follows the file.
GltModel* make_model(GltModelConfig* cfg, int batch, int seq_len, const std::string& st_path) {
  int found = 0;
  int64_t shape[8];
  int nd = 0;
  CHECK(glt_safetensors_tensor_info(st_path.c_str(), "lm_head.weight", &found, shape, &nd));
  cfg->tie_embeddings = found ? 0 : 1;
  if (!found) std::cout << "  lm_head.weight not found -- tying with embed_tokens.weight\n";
  GltModel* m = nullptr;
  CHECK(glt_model_create(cfg, batch, seq_len, GLT_MODEL_DECODER, &m));
  std::cout << "[Component 1] Loading weights (bfloat16) from " << st_path << "\n";
  CHECK(glt_model_load_safetensors(m, st_path.c_str(), nullptr));
  return m;
}

void print_eval(const GltEvalStats& ev) {
  std::cout << "tokens=" << ev.tokens << "\n";
  std::cout << "mean_ce=" << std::setprecision(10) << ev.mean_ce << "\n";
  std::cout << "ppl=" << std::setprecision(10) << ev.ppl << "\n";
  std::cout << "logits_sum=" << std::setprecision(10) << ev.logits_sum << "\n";
  std::cout << "logits_l2=" << std::setprecision(10) << ev.logits_l2 << "\n";
  std::cout << "logits_hash=" << std::hex << ev.logits_hash << std::dec << "\n";
}

int run(int argc, char** argv) {
  GltModelConfig cfg;
  CHECK(glt_config_default(&cfg));
  std::string safetensors_path, domain_data_path, output_path, checkpoint_path, parity_dump_dir;
  std::vector<std::string> ood_data_paths;
  std::string init_deltas_path, eval_data_path, session_id, save_state_path, resume_state_path;
  std::string backend = "rocblas", layout = "overlay";
  int domain_id = 0, max_domains = 4, steps = 200, batch_size = 16, max_len = 512, seed = 42;
  float lr = 2e-4f;
  int parity_dump_layer = -1;
  int stop_after = 0;
  bool eval_only = false, shadow_eval = false, profile = false, contract_probe = false, verbose = false;
  std::vector<int> no_rope;

  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    const bool nx = i + 1 < argc;
    if (a == "--safetensors" && nx) safetensors_path = argv[++i];
    else if (a == "--domain-data" && nx) domain_data_path = argv[++i];
    else if (a == "--ood-data") {
      while (i + 1 < argc && argv[i + 1][0] != '-') ood_data_paths.push_back(argv[++i]);
    }
    else if (a == "--eval-only") eval_only = true;
    else if (a == "--shadow-eval") shadow_eval = true;
    else if (a == "--eval-data" && nx) eval_data_path = argv[++i];
    else if (a == "--domain-id" && nx) domain_id = std::stoi(argv[++i]);
    else if (a == "--max-domains" && nx) max_domains = std::stoi(argv[++i]);
    else if (a == "--steps" && nx) steps = std::stoi(argv[++i]);
    else if (a == "--lr" && nx) lr = std::stof(argv[++i]);
    else if (a == "--lm-loss-scale" && nx) cfg.lm_loss_scale = std::stof(argv[++i]);
    else if (a == "--lambda-silence" && nx) cfg.lambda_silence = std::stof(argv[++i]);
    else if (a == "--batch-size" && nx) batch_size = std::stoi(argv[++i]);
    else if (a == "--max-len" && nx) max_len = std::stoi(argv[++i]);
    else if (a == "--output" && nx) output_path = argv[++i];
    else if (a == "--checkpoint" && nx) checkpoint_path = argv[++i];
    else if (a == "--session-id" && nx) session_id = argv[++i];
    else if (a == "--seed" && nx) seed = std::stoi(argv[++i]);
    else if (a == "--hidden-dim" && nx) cfg.hidden_dim = std::stoi(argv[++i]);
    else if (a == "--intermediate-dim" && nx) cfg.intermediate_dim = std::stoi(argv[++i]);
    else if (a == "--vocab-size" && nx) cfg.vocab_size = std::stoi(argv[++i]);
    else if (a == "--num-layers" && nx) cfg.num_layers = std::stoi(argv[++i]);
    else if (a == "--num-heads" && nx) cfg.num_heads = std::stoi(argv[++i]);
    else if (a == "--num-kv-heads" && nx) cfg.num_kv_heads = std::stoi(argv[++i]);
    else if (a == "--head-dim" && nx) cfg.head_dim = std::stoi(argv[++i]);
    else if (a == "--slice-dim" && nx) cfg.slice_dim = std::stoi(argv[++i]);
    else if (a == "--rope-theta" && nx) cfg.rope_theta = std::stof(argv[++i]);
    else if (a == "--no-rope-layers" && nx) {
      const std::string v = argv[++i];
      size_t pos = 0;
      while (pos < v.size()) {
        const size_t comma = v.find(',', pos);
        const std::string tok = v.substr(pos, comma - pos);
        if (!tok.empty()) no_rope.push_back(std::stoi(tok));
        pos = comma == std::string::npos ? v.size() : comma + 1;
      }
    }
    else if (a == "--beta1" && nx) cfg.adam_beta1 = std::stof(argv[++i]);
    else if (a == "--beta2" && nx) cfg.adam_beta2 = std::stof(argv[++i]);
    else if (a == "--adam-eps" && nx) cfg.adam_eps = std::stof(argv[++i]);
    else if (a == "--weight-decay" && nx) cfg.adam_weight_decay = std::stof(argv[++i]);
    else if (a == "--grad-clip" && nx) cfg.gradient_clip_norm = std::stof(argv[++i]);
    else if (a == "--warmup-steps" && nx) cfg.lr_warmup_steps = std::stoi(argv[++i]);
    else if (a == "--threads" && nx) ++i;  // launch shapes are fixed per kernel here
    else if (a == "--graft-layer-start" && nx) cfg.graft_layer_start = std::stoi(argv[++i]);
    else if (a == "--graft-layer-end" && nx) cfg.graft_layer_end = std::stoi(argv[++i]);
    else if (a == "--graft-proj-gate" && nx) cfg.graft_proj_gate = std::stoi(argv[++i]);
    else if (a == "--graft-proj-up" && nx) cfg.graft_proj_up = std::stoi(argv[++i]);
    else if (a == "--graft-proj-down" && nx) cfg.graft_proj_down = std::stoi(argv[++i]);
    else if (a == "--allow-expansion-trap") cfg.allow_expansion_trap = 1;
    else if (a == "--graft-gemm-backend" && nx) backend = argv[++i];
    else if (a == "--delta-bf16-mirror") {}          // the bf16 graft copy is always kept
    else if (a == "--use-aten-delta-input-grad") {}  // one GEMM path computes every input grad
    else if (a == "--profile-graft-gemms") profile = true;
    else if (a == "--parity-dump" && nx) parity_dump_dir = argv[++i];
    else if (a == "--parity-dump-layer" && nx) parity_dump_layer = std::stoi(argv[++i]);
    else if (a == "--init-deltas" && nx) init_deltas_path = argv[++i];
    else if (a == "--contract-probe") contract_probe = true;
    else if (a == "--verbose") verbose = true;
    else if (a == "--graft-layout" && nx) layout = argv[++i];
    else if (a == "--save-state" && nx) save_state_path = argv[++i];
    else if (a == "--resume-state" && nx) resume_state_path = argv[++i];
    else if (a == "--stop-after" && nx) stop_after = std::stoi(argv[++i]);
    else if (a == "--help") {
      print_usage(argv[0]);
      return 0;
    }
  }
  (void)verbose;
  (void)parity_dump_layer;
  cfg.lr_peak = lr;
  cfg.max_domains = max_domains;
  cfg.domain_id = domain_id;

  // shared validation (grafting.hip:364-444), before any division
  if (cfg.num_heads <= 0) { std::cerr << "Error: --num-heads must be positive.\n"; return EXIT_FAILURE; }
  if (max_domains <= 0) { std::cerr << "Error: --max-domains must be positive.\n"; return EXIT_FAILURE; }
  if (backend != "rocblas" && backend != "hipblaslt-selective") {
    std::cerr << "Error: invalid --graft-gemm-backend '" << backend
              << "' (expected rocblas or hipblaslt-selective)\n";
    return EXIT_FAILURE;
  }
  if (layout == "overlay") cfg.layout = GLT_LAYOUT_OVERLAY;
  else if (layout == "concat") cfg.layout = GLT_LAYOUT_CONCAT;
  else { std::cerr << "Error: invalid --graft-layout '" << layout << "' (expected overlay or concat)\n"; return EXIT_FAILURE; }
  if (!no_rope.empty()) {
    if (no_rope.size() > 256) { std::cerr << "Error: too many --no-rope-layers values.\n"; return EXIT_FAILURE; }
    cfg.no_rope_mask_len = static_cast<int>(no_rope.size());
    for (size_t k = 0; k < no_rope.size(); ++k) cfg.no_rope_mask[k] = no_rope[k];
  }
  if (!parity_dump_dir.empty()) std::system(("mkdir -p '" + parity_dump_dir + "'").c_str());
  if (glt_config_validate(&cfg, batch_size, 1) != GLT_OK) {
    std::cerr << "Error: " << glt_last_error() << "\n";
    return EXIT_FAILURE;
  }
  const int head_dim = cfg.head_dim ? cfg.head_dim : cfg.hidden_dim / cfg.num_heads;
  const int H = cfg.layout == GLT_LAYOUT_CONCAT ? cfg.hidden_dim : cfg.hidden_dim / max_domains;
  const int S = cfg.slice_dim;
  const int64_t graft_numel = static_cast<int64_t>(3) * cfg.num_layers * S * H;
  const char* sid = session_id.empty() ? nullptr : session_id.c_str();

  // training-state flags (new): refused before any device work
  const bool state_flags = !save_state_path.empty() || !resume_state_path.empty() || stop_after != 0;
  if ((eval_only || shadow_eval) && state_flags) {
    std::cerr << "Error: --save-state, --resume-state and --stop-after are training-only.\n";
    return EXIT_FAILURE;
  }
  if (stop_after < 0) {
    std::cerr << "Error: --stop-after must be positive.\n";
    return EXIT_FAILURE;
  }
  if (!resume_state_path.empty() && (!checkpoint_path.empty() || !init_deltas_path.empty())) {
    std::cerr << "Error: --resume-state restores the graft itself; it is incompatible with --checkpoint "
                 "and --init-deltas.\n";
    return EXIT_FAILURE;
  }
  if (!resume_state_path.empty() && !exists(resume_state_path)) {
    std::cerr << "Error: training state '" << resume_state_path << "' does not exist.\n";
    return EXIT_FAILURE;
  }
  if (!save_state_path.empty()) {
    const std::string parent = parent_of(save_state_path);
    if (is_dir(save_state_path) || (!parent.empty() && !exists(parent))) {
      std::cerr << "Error: --save-state path '" << save_state_path
                << "' is a directory or its parent directory does not exist.\n";
      return EXIT_FAILURE;
    }
  }

  // ------------------------------ shadow eval ------------------------------
  if (shadow_eval) {
    if (!domain_data_path.empty()) { std::cerr << "Error: --shadow-eval is incompatible with --domain-data (training-only).\n"; return EXIT_FAILURE; }
    if (!ood_data_paths.empty()) { std::cerr << "Error: --shadow-eval is incompatible with --ood-data (training-only).\n"; return EXIT_FAILURE; }
    if (!output_path.empty()) { std::cerr << "Error: --shadow-eval does not save a checkpoint; remove --output.\n"; return EXIT_FAILURE; }
    if (!init_deltas_path.empty()) { std::cerr << "Error: --shadow-eval is incompatible with --init-deltas (training-only).\n"; return EXIT_FAILURE; }
    if (contract_probe) { std::cerr << "Error: --shadow-eval is incompatible with --contract-probe.\n"; return EXIT_FAILURE; }
    if (safetensors_path.empty() || eval_data_path.empty()) {
      std::cerr << "Error: --shadow-eval requires --safetensors and --eval-data.\n";
      print_usage(argv[0]);
      return EXIT_FAILURE;
    }
    Tokens ev;
    if (!load_bin(eval_data_path, &ev)) return EXIT_FAILURE;
    GltModel* m = make_model(&cfg, batch_size, ev.seq_len, safetensors_path);
    int64_t arena = 0, graft = 0;
    CHECK(glt_model_memory(m, &arena, &graft));
    std::cout << "[Arena] Allocated " << arena / 1024 / 1024 << " MB of VRAM.\n";
    const bool has_ckpt = !checkpoint_path.empty();
    if (has_ckpt) {
      std::cout << "[Checkpoint] Loading graft from " << checkpoint_path << "\n";
      if (glt_model_load_checkpoint(m, checkpoint_path.c_str(), sid, domain_id) != GLT_OK) {
        std::cerr << "Error: " << glt_last_error() << "\n";
        return EXIT_FAILURE;
      }
      CHECK(glt_model_shadow_bake(m, nullptr));
      std::cout << "[Shadow] Graft freed before first forward: yes\n";
    } else {
      std::cout << "[Shadow] Base-only mode (no checkpoint).\n";
    }
    GltEvalStats st;
    CHECK(glt_model_eval(m, ev.tokens.data(), ev.num_sequences, 1, 0, &st, nullptr));
    std::cout << "mode=" << (has_ckpt ? "shadow" : "base") << "\n";
    std::cout << "checkpoint=" << (has_ckpt ? checkpoint_path : "<none>") << "\n";
    print_eval(st);
    std::cout << "shadow_baked=" << (has_ckpt ? "true" : "false") << "\n";
    std::cout << "graft_freed_before_forward=" << (has_ckpt ? "true" : "n/a") << "\n";
    std::cout << "[eval] graft forward calls=" << st.graft_forward_calls
              << " (nonzero = explicit graft GEMMs active)\n";
    glt_model_destroy(m);
    return EXIT_SUCCESS;
  }

  // ------------------------------- eval only -------------------------------
  if (eval_only) {
    bool bad = false;
    if (!domain_data_path.empty()) { std::cerr << "Error: --eval-only is incompatible with --domain-data (training-only).\n"; bad = true; }
    if (!ood_data_paths.empty()) { std::cerr << "Error: --eval-only is incompatible with --ood-data (training-only).\n"; bad = true; }
    if (!output_path.empty()) { std::cerr << "Error: --eval-only does not save a checkpoint; remove --output.\n"; bad = true; }
    if (!init_deltas_path.empty()) { std::cerr << "Error: --eval-only is incompatible with --init-deltas (training-only).\n"; bad = true; }
    if (contract_probe) { std::cerr << "Error: --eval-only is incompatible with --contract-probe.\n"; bad = true; }
    if (bad) return EXIT_FAILURE;
    if (safetensors_path.empty() || eval_data_path.empty()) {
      std::cerr << "Error: --eval-only requires --safetensors and --eval-data.\n";
      print_usage(argv[0]);
      return EXIT_FAILURE;
    }
    Tokens ev;
    if (!load_bin(eval_data_path, &ev)) return EXIT_FAILURE;
    GltModel* m = make_model(&cfg, batch_size, ev.seq_len, safetensors_path);
    int64_t arena = 0, graft = 0;
    CHECK(glt_model_memory(m, &arena, &graft));
    std::cout << "[Arena] Allocated " << arena / 1024 / 1024 << " MB of VRAM.\n";
    bool active = false;
    if (!checkpoint_path.empty()) {
      std::cout << "[Checkpoint] Loading graft from " << checkpoint_path << "\n";
      if (glt_model_load_checkpoint(m, checkpoint_path.c_str(), sid, domain_id) != GLT_OK) {
        std::cerr << "Error: " << glt_last_error() << "\n";
        return EXIT_FAILURE;
      }
      active = true;
    }
    std::cout << "graft.active=" << (active ? "true" : "false") << std::endl;
    GltEvalStats st;
    CHECK(glt_model_eval(m, ev.tokens.data(), ev.num_sequences, 1, active ? 1 : 0, &st, nullptr));
    std::cout << "mode=" << (active ? "grafted" : "base") << "\n";
    std::cout << "checkpoint=" << (checkpoint_path.empty() ? "<none>" : checkpoint_path) << "\n";
    print_eval(st);
    std::cout << "[eval] graft forward calls=" << st.graft_forward_calls << " (expected 0 for base-only)\n";
    glt_model_destroy(m);
    return EXIT_SUCCESS;
  }

  // -------------------------------- training -------------------------------
  if (safetensors_path.empty() || domain_data_path.empty() || ood_data_paths.empty() || output_path.empty()) {
    std::cerr << "Error: --safetensors, --domain-data, --ood-data (at least one), and --output are required.\n";
    print_usage(argv[0]);
    return EXIT_FAILURE;
  }
  if (is_dir(output_path)) {
    std::cerr << "Error: --output path '" << output_path << "' is a directory. "
              << "Specify a file path (e.g., /path/to/checkpoint.safetensors).\n";
    return EXIT_FAILURE;
  }
  {
    const std::string parent = parent_of(output_path);
    if (!parent.empty() && !exists(parent)) {
      std::cerr << "Error: parent directory '" << parent << "' does not exist.\n";
      return EXIT_FAILURE;
    }
  }
  if (glt_config_validate(&cfg, batch_size, 0) != GLT_OK) {
    std::cerr << "Error: " << glt_last_error() << "\n";
    return EXIT_FAILURE;
  }
  Tokens domain, ood;
  if (!load_bin(domain_data_path, &domain)) return EXIT_FAILURE;
  if (domain.num_sequences == 0) {
    std::cerr << "Error: domain data file '" << domain_data_path << "' has 0 sequences.\n";
    return EXIT_FAILURE;
  }
  for (const auto& p : ood_data_paths) {
    Tokens t;
    if (!load_bin(p, &t)) return EXIT_FAILURE;
    if (t.num_sequences == 0) {
      std::cerr << "Warning: OOD file '" << p << "' has 0 sequences -- skipping.\n";
      continue;
    }
    if (t.seq_len != domain.seq_len) {
      std::cerr << "Error: seq_len mismatch. Domain has " << domain.seq_len << ", OOD file " << p
                << " has " << t.seq_len << "\n";
      return EXIT_FAILURE;
    }
    ood.tokens.insert(ood.tokens.end(), t.tokens.begin(), t.tokens.end());
    ood.num_sequences += t.num_sequences;
  }
  if (ood.num_sequences == 0) {
    std::cerr << "Error: no valid OOD sequences loaded.\n";
    return EXIT_FAILURE;
  }
  ood.seq_len = domain.seq_len;
  if (max_len != domain.seq_len)
    std::cerr << "Warning: --max-len (" << max_len << ") != file seq_len (" << domain.seq_len
              << "). Using file value.\n";
  const int T = domain.seq_len;

  std::cout << "=== Grafting Training Binary ===\n";
  std::cout << "Model: " << cfg.hidden_dim << "hd " << cfg.num_layers << "L " << cfg.num_heads << "h "
            << cfg.num_kv_heads << "kvh " << head_dim << "d " << cfg.vocab_size << "voc\n";
  if (cfg.layout == GLT_LAYOUT_OVERLAY)
    std::cout << "Domain ID: " << domain_id << " / " << max_domains << " (I-slice: " << domain_id * S
              << " to " << (domain_id + 1) * S << ", H-slice: " << domain_id * H << " to "
              << (domain_id + 1) * H << ")\n";
  else
    std::cout << "Graft layout: concat (" << S << " graft columns after " << cfg.intermediate_dim
              << " base columns, H = hidden)\n";
  int active = 0;
  for (int l = 0; l < cfg.num_layers; ++l)
    if (l >= cfg.graft_layer_start && l <= cfg.graft_layer_end)
      active += cfg.graft_proj_gate + cfg.graft_proj_up + cfg.graft_proj_down;
  std::cout << "Graft projections: gate=" << cfg.graft_proj_gate << ", up=" << cfg.graft_proj_up
            << ", down=" << cfg.graft_proj_down << ", active_grafts=" << active << "\n";
  std::cout << "Domain sequences: " << domain.num_sequences << ", OOD sequences: " << ood.num_sequences << "\n";
  std::cout << "Seq len: " << T << ", Batch size: " << batch_size << ", Steps: " << steps << ", LR: " << lr
            << ", LM loss scale: " << cfg.lm_loss_scale << ", Lambda silence: " << cfg.lambda_silence << "\n";
  std::cout << "Seed: " << seed << "\n";

  GltModel* m = make_model(&cfg, batch_size, T, safetensors_path);
  int64_t peak_mb = used_mb();
  {
    int64_t arena = 0, graft = 0;
    CHECK(glt_model_memory(m, &arena, &graft));
    std::cout << "[Arena] Allocated " << arena / 1024 / 1024 << " MB of VRAM.\n";
  }
  float *d_w = nullptr, *d_g = nullptr, *d_m = nullptr, *d_v = nullptr;
  int64_t n = 0;
  CHECK(glt_model_graft_buffers(m, &d_w, &d_g, &d_m, &d_v, &n));
  if (n != graft_numel) throw GltFailure("graft size mismatch");

  if (!checkpoint_path.empty()) {
    std::cout << "[Checkpoint] Loading from " << checkpoint_path << "\n";
    if (glt_model_load_checkpoint(m, checkpoint_path.c_str(), sid, domain_id) != GLT_OK) {
      std::cerr << "Error: " << glt_last_error() << "\n";
      return EXIT_FAILURE;
    }
  }
  if (!init_deltas_path.empty()) {  // grafting.hip:883-915
    std::cout << "[Parity] Loading initial deltas from " << init_deltas_path << "\n";
    const size_t expected = static_cast<size_t>(graft_numel) * sizeof(float);
    std::ifstream f(init_deltas_path, std::ios::binary | std::ios::ate);
    if (!f) { std::cerr << "Error: cannot open " << init_deltas_path << "\n"; return EXIT_FAILURE; }
    const size_t bytes = static_cast<size_t>(f.tellg());
    if (bytes != expected) {
      std::cerr << "Error: " << init_deltas_path << " size " << bytes << " != expected " << expected << "\n";
      return EXIT_FAILURE;
    }
    std::vector<float> host(static_cast<size_t>(graft_numel));
    f.seekg(0);
    f.read(reinterpret_cast<char*>(host.data()), static_cast<std::streamsize>(expected));
    CHECK(glt_memcpy(d_w, host.data(), static_cast<int64_t>(expected), nullptr, 1));
    std::vector<float> zeros(host.size(), 0.f);
    CHECK(glt_memcpy(d_m, zeros.data(), static_cast<int64_t>(expected), nullptr, 1));
    CHECK(glt_memcpy(d_v, zeros.data(), static_cast<int64_t>(expected), nullptr, 1));
    CHECK(glt_model_refresh_graft(m, nullptr));
    std::cout << "[Parity] Loaded " << host.size() << " floats. Adam states zeroed.\n";
    if (!parity_dump_dir.empty()) write_raw(parity_dump_dir + "/delta_weights_loaded.raw", host.data(), expected);
  }

  int start_step = 0;
  if (!resume_state_path.empty()) {
    int64_t k = 0;
    std::cout << "[State] Resuming from " << resume_state_path << "\n";
    if (glt_model_load_train_state(m, resume_state_path.c_str(), sid, domain_id, &k) != GLT_OK) {
      std::cerr << "Error: " << glt_last_error() << "\n";
      return EXIT_FAILURE;
    }
    if (k >= steps) {
      std::cerr << "Error: the training state is at step " << k << "; --steps " << steps
                << " is the length of the schedule and leaves nothing to run.\n";
      return EXIT_FAILURE;
    }
    start_step = static_cast<int>(k);
    std::cout << "[State] Restored the fp32 graft, the Adam moments and step " << k << ".\n";
  }
  const int end_step = stop_after > 0 ? std::min(steps, stop_after) : steps;
  if (end_step <= start_step) {
    std::cerr << "Error: --stop-after " << stop_after << " leaves nothing to run from step " << start_step << ".\n";
    return EXIT_FAILURE;
  }

  if (contract_probe) {  // run_contract_sparse_probe (graft_ops_impl.inc:158-212)
    std::cout << "[ContractProbe] Running synthetic sparse contract-forward test.\n";
    const int M = 2, stride = cfg.intermediate_dim;
    std::vector<uint16_t> x(static_cast<size_t>(M) * stride, 0);
    std::vector<float> w(static_cast<size_t>(S) * H, 0.f), out(static_cast<size_t>(M) * H, 0.f);
    x[3] = 0x4000;                 // 2.0 in bf16
    x[stride + 17] = 0xC0A0;       // -5.0
    if (S > 29 && H > 31) {
      w[3 * H + 11] = 7.f;
      w[17 * H + 23] = -13.f;
      w[29 * H + 31] = 19.f;
    }
    void *dx = nullptr, *dw = nullptr, *dout = nullptr;
    CHECK(glt_malloc(&dx, static_cast<int64_t>(x.size()) * 2));
    CHECK(glt_malloc(&dw, static_cast<int64_t>(w.size()) * 4));
    CHECK(glt_malloc(&dout, static_cast<int64_t>(out.size()) * 4));
    CHECK(glt_memcpy(dx, x.data(), static_cast<int64_t>(x.size()) * 2, nullptr, 0));
    CHECK(glt_memcpy(dw, w.data(), static_cast<int64_t>(w.size()) * 4, nullptr, 0));
    GltArena* ar = nullptr;
    CHECK(glt_arena_create(64ll << 20, &ar));
    CHECK(glt_graft_op(GLT_GRAFT_CONTRACT_FWD, M, S, H, static_cast<const float*>(dw), nullptr, dx, 0,
                       stride, nullptr, 0, 0, static_cast<float*>(dout), H, 1.f, 0.f, ar, nullptr));
    CHECK(glt_memcpy(out.data(), dout, static_cast<int64_t>(out.size()) * 4, nullptr, 1));
    std::cout << "[ContractProbe] synthetic sparse mapping results:\n";
    float max_abs = 0.f;
    int mm = -1, mh = -1;
    for (int r = 0; r < M; ++r)
      for (int h = 0; h < H; ++h) {
        const float v = out[static_cast<size_t>(r) * H + h];
        if (std::fabs(v) > max_abs) { max_abs = std::fabs(v); mm = r; mh = h; }
        if (std::fabs(v) > 1e-7f) std::cout << "  out[" << r << "," << h << "]=" << v << "\n";
      }
    std::cout << "[ContractProbe] max_abs=" << max_abs << " at out[" << mm << "," << mh << "]="
              << (mm >= 0 ? out[static_cast<size_t>(mm) * H + mh] : 0.f) << "\n";
    std::cout << "[ContractProbe] expected: out[0,11]=14, out[1,23]=65, others ~0\n";
    glt_arena_destroy(ar);
    glt_free(dx);
    glt_free(dw);
    glt_free(dout);
    glt_model_destroy(m);
    return 0;
  }

  // grafting.hip:932-933: everything before the last '.', then "_log.csv"
  const std::string log_path = output_path.substr(0, output_path.find_last_of('.')) + "_log.csv";
  // a resumed run appends to the log of the run it continues
  const bool fresh_log = start_step == 0 || file_size(log_path) <= 0;
  std::ofstream log_file(log_path, fresh_log ? std::ios::trunc : std::ios::app);
  if (log_file && fresh_log)
    log_file << "step,lm_loss,silence_loss,domain_graft_energy,ood_graft_energy,domain_ood_energy_ratio,"
                "total_loss,lr,grad_norm,step_time_sec\n";
  if (start_step)
    std::cout << "[Loop] Resuming training at step " << start_step << " of " << steps
              << ".\n       Logging to " << log_path << "\n";
  else
    std::cout << "[Loop] Starting training for " << steps << " steps.\n       Logging to " << log_path << "\n";
  if (profile) CHECK(glt_model_profile(m, 1));

  int dpos = 0, opos = 0;
  CHECK(glt_batch_walk_start(static_cast<uint64_t>(static_cast<int64_t>(seed)), domain.num_sequences,
                             ood.num_sequences, &dpos, &opos));
  std::vector<int32_t> ids(static_cast<size_t>(batch_size) * T), mask(ids.size());
  std::vector<double> steady;
  float prev_norm = -1.f;
  for (int s = 0; s < start_step; ++s)  // the data walk of the steps already taken
    CHECK(glt_batch_step(domain.tokens.data(), domain.num_sequences, ood.tokens.data(), ood.num_sequences, T,
                         batch_size, &dpos, &opos, ids.data(), mask.data()));
  // Logs one finished step (CSV line, parity dump at step 0, console line).
  auto log_step = [&](int step, const GltStepStats& st, double sec) {
    peak_mb = std::max(peak_mb, used_mb());
    if (step > start_step) steady.push_back(sec);
    // The reference logs the previous step's clip coefficient read back
    // asynchronously: grad_norm = clip / scale, scale = norm > clip ? clip / norm : 1
    // (calc_scale_kernel, kernels_elementwise_impl.inc:167-196), -1 at step 0.
    float grad_norm = -1.f, host_scale = -1.f;
    if (step > start_step) {
      host_scale = prev_norm > cfg.gradient_clip_norm ? cfg.gradient_clip_norm / prev_norm : 1.f;
      grad_norm = host_scale > 0.f ? cfg.gradient_clip_norm / host_scale : 0.f;
    }
    prev_norm = st.grad_norm;
    if (log_file)
      log_file << step << "," << st.lm_loss << "," << st.silence_loss << "," << st.domain_graft_energy << ","
               << st.ood_graft_energy << "," << st.domain_ood_energy_ratio << "," << st.total_loss << ","
               << st.lr << "," << grad_norm << "," << sec << "\n";
    if (step == 0 && !parity_dump_dir.empty()) {  // grafting.hip:1207-1245
      const std::string pd = parity_dump_dir + "/";
      std::ofstream lf(pd + "losses.csv");
      lf << "lm_loss,silence_loss,domain_graft_energy,ood_graft_energy,domain_ood_energy_ratio,total_loss,grad_norm,step_time_sec\n";
      lf << st.lm_loss << "," << st.silence_loss << "," << st.domain_graft_energy << "," << st.ood_graft_energy << ","
         << st.domain_ood_energy_ratio << "," << st.total_loss << "," << grad_norm << "," << sec << "\n";
      std::ofstream(pd + "grad_clip_coef.txt") << host_scale << "\n";
      std::ofstream(pd + "lm_loss.txt") << st.lm_loss << "\n";
      std::vector<float> host(static_cast<size_t>(graft_numel));
      // the reference dumps the gradients after clipping (apply_scale_kernel)
      CHECK(glt_memcpy(host.data(), d_g, graft_numel * 4, nullptr, 1));
      const float sc = st.grad_norm > cfg.gradient_clip_norm ? cfg.gradient_clip_norm / st.grad_norm : 1.f;
      for (float& g : host) g *= sc;
      write_raw(pd + "delta_grads.raw", host.data(), host.size() * 4);
      CHECK(glt_memcpy(host.data(), d_w, graft_numel * 4, nullptr, 1));
      write_raw(pd + "delta_weights_post.raw", host.data(), host.size() * 4);
    }
    if (step % 50 == 0)
      std::cout << "  Step " << step << "/" << steps << " | lm=" << st.lm_loss << " | silence=" << st.silence_loss
                << " | total=" << st.total_loss << " | lr=" << st.lr << " | grad_norm=" << grad_norm << "\n";
  };
  // Steps are enqueued one ahead of the logging: the device runs step k+1
  // while the host reads and logs step k (glt_model_step_stats), so no host
  // sync stalls the device between steps; a step's time is the interval
  // between consecutive step completions.  The parity dump reads step 0's
  // gradients before step 1 may run, so with it every step is synchronous.
  const bool pipelined = parity_dump_dir.empty();
  auto t_prev = std::chrono::steady_clock::now();
  for (int step = start_step; step < end_step; ++step) {
    CHECK(glt_batch_step(domain.tokens.data(), domain.num_sequences, ood.tokens.data(), ood.num_sequences, T,
                         batch_size, &dpos, &opos, ids.data(), mask.data()));
    GltStepStats st;
    if (pipelined) {
      CHECK(glt_train_step(m, ids.data(), mask.data(), 1, step, steps, nullptr, nullptr));
      if (step > start_step) {
        CHECK(glt_model_step_stats(m, step - 1, &st));
        const auto now = std::chrono::steady_clock::now();
        const double sec = std::chrono::duration<double>(now - t_prev).count();
        t_prev = now;
        log_step(step - 1, st, sec);
      }
    } else {
      const auto t0 = std::chrono::steady_clock::now();
      CHECK(glt_train_step(m, ids.data(), mask.data(), 1, step, steps, &st, nullptr));
      log_step(step, st, std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
    }
  }
  if (pipelined) {
    GltStepStats st;
    CHECK(glt_model_step_stats(m, end_step - 1, &st));
    const double sec = std::chrono::duration<double>(std::chrono::steady_clock::now() - t_prev).count();
    log_step(end_step - 1, st, sec);
  }
  double p50 = 0.0;
  if (!steady.empty()) {
    std::vector<double> tmp = steady;
    std::sort(tmp.begin(), tmp.end());
    const size_t k = tmp.size() / 2;
    p50 = tmp.size() % 2 ? tmp[k] : (tmp[k - 1] + tmp[k]) / 2.0;
  }
  std::cout << "sec_per_step_p50=" << std::fixed << std::setprecision(6) << p50 << "\n";
  std::cout << "peak_train_vram_mb=" << peak_mb << "\n";
  std::cout << "timed_steps=" << steady.size() << "\n";
  std::cout << "warmup_steps_excluded=1\n";
  std::cout.unsetf(std::ios::fixed);
  std::cout << "[Save] Writing safetensors to " << output_path << "\n";
  CHECK(glt_model_save_checkpoint(m, output_path.c_str(), session_id.c_str(), domain_id));
  if (!save_state_path.empty()) {
    std::cout << "[State] Writing the training state (step " << end_step << ") to " << save_state_path << "\n";
    CHECK(glt_model_save_train_state(m, save_state_path.c_str(), session_id.c_str(), domain_id, end_step));
  }
  if (profile) {  // write_gemm_profile_stats_json (checkpoint_impl.inc:107-168), per fused kernel kind
    double ms[GLT_PROF_KINDS];
    int64_t calls[GLT_PROF_KINDS];
    CHECK(glt_model_profile_read(m, ms, calls, 0));
    std::ofstream f(replace_ext(output_path, ".graft_gemm_stats.json"));
    f << "{\n  \"graft_gemm_backend\": \"tcgen05\",\n  \"requested_backend\": \"" << backend
      << "\",\n  \"stats\": {\n";
    for (int k = 0; k < GLT_PROF_KINDS; ++k)
      f << "    \"" << kProfNames[k] << "\": {\"call_count\":" << calls[k] << ",\"total_ms\":" << ms[k]
        << ",\"backend\":\"tcgen05\"}" << (k + 1 < GLT_PROF_KINDS ? "," : "") << "\n";
    f << "  }\n}\n";
  }
  glt_model_destroy(m);
  std::cout << "Experiment completed successfully.\n";
  return EXIT_SUCCESS;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    return run(argc, argv);
  } catch (const std::exception& e) {
    std::cerr << "Fatal: " << e.what() << "\n";
    return EXIT_FAILURE;
  }
}
