// SPDX-License-Identifier: 0BSD

//go:build cuda

package infer

import (
	"os"
	"testing"

	"quad4.io/auto-commit-msg/internal/gguf"
)

// The CUDA build through the app's own calls (app.go:253-287): Load from the
// parsed file, greedy Generate, Stats, Reset, and Forward agreeing with
// Generate's first id.  ACM_TEST_GGUF names a model file (any qwen2/qwen3/
// llama GGUF; the repository's synth.py writes seeded ones).
func TestCUDAGenerate(t *testing.T) {
	path := os.Getenv("ACM_TEST_GGUF")
	if path == "" {
		t.Skip("ACM_TEST_GGUF not set")
	}
	data, err := os.ReadFile(path)
	if err != nil {
		t.Fatal(err)
	}
	f, err := gguf.Parse(data)
	if err != nil {
		t.Fatal(err)
	}
	m, err := Load(f, 512)
	if err != nil {
		t.Fatal(err)
	}
	defer m.Close()
	prompt := []int{m.Cfg.BOS, 11, 12, 13, 14, 15, 16, 17}
	logits, err := m.Forward(prompt)
	if err != nil {
		t.Fatal(err)
	}
	first := MaxLogit(logits)
	if m.Pos() != len(prompt) {
		t.Fatalf("pos %d, want %d", m.Pos(), len(prompt))
	}
	m.Reset()
	ids, err := m.Generate(prompt, &Sampler{}, 16, nil)
	if err != nil {
		t.Fatal(err)
	}
	if len(ids) == 0 || ids[0] != first {
		t.Fatalf("generate %v, forward's greedy id %d", ids, first)
	}
	if m.Stats.PrefillToks != len(prompt) || m.Stats.DecodeToks != len(ids) {
		t.Fatalf("stats %+v for %d ids", m.Stats, len(ids))
	}
	// the context limit is the reference's error
	m.Reset()
	long := make([]int, 600)
	if _, err := m.Forward(long); err == nil {
		t.Fatal("600 tokens at ctx 512: no error")
	}
}
