// SPDX-License-Identifier: 0BSD

//go:build cuda

// Package infer, CUDA build: the reference's exported inference API
// (internal/infer/model.go:14-471, sampler.go:12-157) served by
// libacmcuda.so through its C ABI (include/acm.h).  With the `cuda` tag this
// file replaces model.go, tensor.go, sampler.go, dot.go and the dispatch /
// dequant files, which then carry `//go:build !cuda`; app.Generate
// (internal/app/app.go:230-308) compiles unchanged against it.
//
// The one change outside this package: gguf.File keeps the bytes it was
// parsed from (a `Raw []byte` field that gguf.Parse sets), so Load can hand
// the mapping to the library, which applies gguf.Parse and infer.Load's
// rules itself (same checks, same error texts) and uploads the blocks
// unchanged.
package infer

/*
#cgo CFLAGS: -I${SRCDIR}/../../third_party/acm/include
#cgo LDFLAGS: -L${SRCDIR}/../../third_party/acm/lib -lacmcuda -Wl,-rpath,${SRCDIR}/../../third_party/acm/lib
#include <stdlib.h>
#include "acm.h"
*/
import "C"

import (
	"errors"
	"fmt"
	"math/rand"
	"runtime"
	"sync"
	"time"
	"unsafe"

	"quad4.io/auto-commit-msg/internal/gguf"
)

// Config mirrors model.go:14-40 field for field (app.go reads Arch and BOS).
type Config struct {
	Arch            string
	NLayers         int
	NEmbd           int
	NHead           int
	NHeadKV         int
	HeadDim         int
	NFF             int
	Vocab           int
	MaxCtx          int
	RopeDim         int
	RopeBase        float32
	RopeInterleaved bool
	RopeScaling     string
	RopeFactor      float32
	RopeLoF         float32
	RopeHiF         float32
	RopeOrigCtx     float32
	RMSEps          float32
	BOS             int
	EOS             int
	EOS2            int
}

// HeadKV as model.go:205-210: kv heads, defaulting to the query heads.
func (c *Config) HeadKV() int {
	if c.NHeadKV > 0 {
		return c.NHeadKV
	}
	return c.NHead
}

// Sampler mirrors sampler.go:12-17.
type Sampler struct {
	Temp float64 // 0 = greedy
	TopK int
	TopP float64
	Rng  *rand.Rand
}

// Stats mirrors sampler.go:101-106.  Durations are device time (CUDA
// events), not wall time.
type Stats struct {
	PrefillToks int
	Prefill     time.Duration
	DecodeToks  int
	Decode      time.Duration
}

// DebugLayer, if non-nil, is called after each Forward with (layer index,
// residual stream after that layer).  Unlike model.go:231-233, x holds only
// the LAST token's row ([embd]) and the calls come after the pass, from the
// library's per-layer copy (acm_model_debug_layers).
var DebugLayer func(li int, x []float32)

// Model is one device-resident model with one sequence (the reference's
// Model holds exactly one).  Call Close to free the device memory; the
// reference's Model is garbage-collected, so a finalizer does it as well.
type Model struct {
	Cfg    Config
	Stats  Stats
	eng    *C.acm_engine
	m      *C.acm_model
	seq    C.int32_t
	logits []float32
	dbg    bool
}

// Device selects the GPU that Load opens (default 0).
var Device = 0

var archNames = map[C.int32_t]string{C.ACM_ARCH_QWEN3: "qwen3", C.ACM_ARCH_QWEN2: "qwen2", C.ACM_ARCH_LLAMA: "llama"}
var scalingNames = map[C.int32_t]string{C.ACM_ROPE_NONE: "", C.ACM_ROPE_LINEAR: "linear", C.ACM_ROPE_LLAMA3: "llama3"}

func goBool(v C.int32_t) bool { return v != 0 }

func cfgFromC(c *C.acm_config) Config {
	return Config{
		Arch: archNames[c.arch], NLayers: int(c.n_layers), NEmbd: int(c.n_embd), NHead: int(c.n_head),
		NHeadKV: int(c.n_head_kv), HeadDim: int(c.head_dim), NFF: int(c.n_ff), Vocab: int(c.vocab),
		MaxCtx: int(c.max_ctx), RopeDim: int(c.rope_dim), RopeBase: float32(c.rope_base),
		RopeInterleaved: goBool(c.rope_interleaved), RopeScaling: scalingNames[c.rope_scaling],
		RopeFactor: float32(c.rope_factor), RopeLoF: float32(c.rope_lo_f), RopeHiF: float32(c.rope_hi_f),
		RopeOrigCtx: float32(c.rope_orig_ctx), RMSEps: float32(c.rms_eps),
		BOS: int(c.bos), EOS: int(c.eos), EOS2: int(c.eos2),
	}
}

func (m *Model) status(rc C.int) error {
	if rc == C.ACM_OK {
		return nil
	}
	return errors.New(C.GoString(C.acm_last_error(m.m)))
}

// Load (model.go:90-203): parse, config rules and tensor checks in the
// library (the reference's error texts), blocks uploaded unchanged.
func Load(f *gguf.File, maxCtx int) (*Model, error) {
	if f == nil || len(f.Raw) == 0 {
		return nil, fmt.Errorf("gguf file holds no bytes")
	}
	mdl := &Model{}
	if rc := C.acm_open(C.int(Device), &mdl.eng); rc != C.ACM_OK {
		return nil, fmt.Errorf("acm_open(%d): status %d", Device, int(rc))
	}
	// f.Raw is the mapping (or the embedded model); the call copies what it
	// needs and keeps no pointer into it.
	rc := C.acm_model_load_gguf_mem(mdl.eng, unsafe.Pointer(&f.Raw[0]), C.size_t(len(f.Raw)),
		C.int32_t(maxCtx), 1, &mdl.m)
	if rc != C.ACM_OK {
		err := errors.New(C.GoString(C.acm_engine_error(mdl.eng)))
		C.acm_close(mdl.eng)
		return nil, err
	}
	var cc C.acm_config
	C.acm_model_config(mdl.m, &cc)
	mdl.Cfg = cfgFromC(&cc)
	mdl.logits = make([]float32, mdl.Cfg.Vocab)
	if err := mdl.status(C.acm_seq_open(mdl.m, &mdl.seq)); err != nil {
		mdl.Close()
		return nil, err
	}
	runtime.SetFinalizer(mdl, (*Model).Close)
	return mdl, nil
}

// Close frees the model's device memory and its engine (no reference
// counterpart).
func (m *Model) Close() {
	if m.m != nil {
		C.acm_model_destroy(m.m)
		m.m = nil
	}
	if m.eng != nil {
		C.acm_close(m.eng)
		m.eng = nil
	}
	runtime.SetFinalizer(m, nil)
}

func cIDs(tokens []int) []C.int32_t {
	ids := make([]C.int32_t, len(tokens))
	for i, t := range tokens {
		ids[i] = C.int32_t(t)
	}
	return ids
}

// Forward (model.go:317-442): runs tokens at positions Pos().. and returns
// the last token's logits, a slice the model owns and the next call
// overwrites (as the reference's scratch logits).
func (m *Model) Forward(tokens []int) ([]float32, error) {
	if len(tokens) == 0 {
		return nil, fmt.Errorf("empty token batch")
	}
	m.debugOn()
	ids := cIDs(tokens)
	rc := C.acm_forward(m.m, m.seq, &ids[0], C.int32_t(len(ids)), (*C.float)(unsafe.Pointer(&m.logits[0])))
	if err := m.status(rc); err != nil {
		return nil, err
	}
	m.debugCall()
	return m.logits, nil
}

func (m *Model) debugOn() {
	want := DebugLayer != nil
	if want != m.dbg {
		C.acm_model_debug_layers(m.m, cBool(want))
		m.dbg = want
	}
}

func (m *Model) debugCall() {
	if DebugLayer == nil {
		return
	}
	L, E := m.Cfg.NLayers, m.Cfg.NEmbd
	buf := make([]float32, L*E)
	if C.acm_model_debug_layers_read(m.m, (*C.float)(unsafe.Pointer(&buf[0])), C.int64_t(len(buf))) != C.ACM_OK {
		return
	}
	for li := 0; li < L; li++ {
		DebugLayer(li, buf[li*E:(li+1)*E])
	}
}

func cBool(b bool) C.int32_t {
	if b {
		return 1
	}
	return 0
}

// Generate (sampler.go:111-157): prefill in chunks of at most 1024 tokens,
// then the decode loop on the device until EOS, EOS2 or maxTok.  onToken is
// called for each generated id after the loop returns (the ids are produced
// on the device); Stats holds the device times.
func (m *Model) Generate(prompt []int, s *Sampler, maxTok int, onToken func(id int)) ([]int, error) {
	if len(prompt) == 0 {
		return nil, fmt.Errorf("empty prompt")
	}
	ids := cIDs(prompt)
	cs := C.acm_sampler{temp: C.double(s.Temp), top_k: C.int32_t(s.TopK), top_p: C.double(s.TopP)}
	if s.Rng != nil {
		// one draw per call keeps app/rand.go's different-every-run behaviour;
		// the library's Philox stream is keyed by it
		cs.seed = C.uint64_t(s.Rng.Uint64())
	}
	out := make([]C.int32_t, maxTok+1)
	var n C.int32_t
	var st C.acm_stats
	rc := C.acm_generate(m.m, m.seq, &ids[0], C.int32_t(len(ids)), &cs, C.int32_t(maxTok), 1, &out[0], &n, &st)
	m.Stats = Stats{PrefillToks: int(st.prefill_toks), Prefill: time.Duration(float64(st.prefill_s) * 1e9),
		DecodeToks: int(st.decode_toks), Decode: time.Duration(float64(st.decode_s) * 1e9)}
	res := make([]int, int(n))
	for i := range res {
		res[i] = int(out[i])
		if onToken != nil {
			onToken(res[i])
		}
	}
	return res, m.status(rc)
}

// Pos (model.go:456): positions held by the sequence.
func (m *Model) Pos() int {
	var p C.int32_t
	C.acm_seq_pos(m.m, m.seq, &p)
	return int(p)
}

// Reset (model.go:460): start a new sequence; the cache pages are kept.
func (m *Model) Reset() { C.acm_seq_reset(m.m, m.seq) }

var (
	sampleMu  sync.Mutex
	sampleEng *C.acm_engine // opened on Device by the first Sample call
)

// Sample (sampler.go:30-78) on host logits, through the library's sampler
// (same rules; the draw is Philox keyed by one Rng draw).  Generate does not
// use it: its sampling stays on the device.
func (s *Sampler) Sample(logits []float32) int {
	cs := C.acm_sampler{temp: C.double(s.Temp), top_k: C.int32_t(s.TopK), top_p: C.double(s.TopP)}
	if s.Rng != nil {
		cs.seed = C.uint64_t(s.Rng.Uint64())
	}
	sampleMu.Lock()
	defer sampleMu.Unlock()
	// Sample has no error result: without the device it fails loudly
	// rather than choosing on the host
	if sampleEng == nil {
		if rc := C.acm_open(C.int(Device), &sampleEng); rc != C.ACM_OK {
			sampleEng = nil
			panic(fmt.Sprintf("infer: CUDA device %d unavailable (status %d)", Device, int(rc)))
		}
	}
	var id C.int32_t
	if rc := C.acm_sample_logits(sampleEng, (*C.float)(unsafe.Pointer(&logits[0])), C.int32_t(len(logits)), &cs, 0,
		&id); rc != C.ACM_OK {
		panic(fmt.Sprintf("infer: sample: %s", C.GoString(C.acm_engine_error(sampleEng))))
	}
	return int(id)
}

// MaxLogit (model.go:462-471): index of the first maximum.
func MaxLogit(logits []float32) int {
	if len(logits) == 0 {
		return 0
	}
	return int(C.acm_max_logit((*C.float)(unsafe.Pointer(&logits[0])), C.int32_t(len(logits))))
}
