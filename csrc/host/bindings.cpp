// Python bindings of the host core: module rs_nanogpt_b200._host.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstring>

#include "bpe.h"
#include "chacha.h"
#include "pack.h"
#include "pretok.h"
#include "render.h"
#include "trainer.h"

namespace py = pybind11;
using namespace nanogpt_host;

template <class T>
static py::array_t<T> to_array(const std::vector<T>& v) {
  py::array_t<T> a(v.size());
  if (!v.empty()) std::memcpy(a.mutable_data(), v.data(), v.size() * sizeof(T));
  return a;
}

static std::vector<uint32_t> ids_from(py::handle h) {
  auto a = py::array_t<uint32_t, py::array::c_style | py::array::forcecast>::ensure(h);
  if (!a) throw std::invalid_argument("expected a sequence of token ids");
  return std::vector<uint32_t>(a.data(), a.data() + a.size());
}

static Conversation conv_from(py::handle obj) {
  Conversation conv;
  for (py::handle m : obj) {
    auto t = m.cast<py::tuple>();
    Message msg;
    msg.role = t[0].cast<int>();
    py::handle content = t[1];
    if (py::isinstance<py::str>(content)) {
      msg.has_parts = false;
      msg.text = content.cast<std::string>();
    } else {
      msg.has_parts = true;
      for (py::handle p : content) {
        auto pt = p.cast<py::tuple>();
        msg.parts.push_back({pt[0].cast<int>(), pt[1].cast<std::string>()});
      }
    }
    conv.push_back(std::move(msg));
  }
  return conv;
}

static py::tuple rendered_to_py(const Rendered& r) {
  return py::make_tuple(to_array(r.ids), to_array(r.mask).attr("astype")("bool"));
}

PYBIND11_MODULE(_host, m) {
  m.doc() = "Host-side C++ core: pre-tokenizer, BPE, trainer, packers, chat render, ChaCha8";

  m.def("pre_tokenize", [](const std::string& text) {
    std::vector<std::pair<uint32_t, uint32_t>> pieces;
    pre_tokenize(text, pieces);
    py::list out;
    for (auto [b, e] : pieces) out.append(py::bytes(text.data() + b, e - b).attr("decode")("utf-8"));
    return out;
  });
  m.def("base64_encode", [](py::bytes b) { return base64_encode(std::string(b)); });

  py::class_<Tokenizer>(m, "Tokenizer")
      .def_static("from_file", &Tokenizer::from_file)
      .def_static("from_merges", [](const std::vector<py::bytes>& merges) {
        std::vector<std::string> ms;
        for (auto& b : merges) ms.emplace_back(std::string(b));
        return Tokenizer::from_merges(ms);
      })
      .def("bos_id", &Tokenizer::bos_id)
      .def("vocab_size", &Tokenizer::vocab_size)
      .def("special_id", [](const Tokenizer& t, const std::string& n) -> py::object {
        int id = t.special_id(n);
        if (id < 0) return py::none();
        return py::int_(id);
      })
      .def("token_bytes", [](const Tokenizer& t, uint32_t id) { return py::bytes(t.token_bytes(id)); })
      .def("token_byte_lengths", [](const Tokenizer& t) { return to_array(t.token_byte_lengths()); })
      .def("encode", [](const Tokenizer& t, const std::string& s) {
        std::vector<uint32_t> ids;
        { py::gil_scoped_release nogil; ids = t.encode(s); }
        return to_array(ids);
      })
      .def("encode_batch", [](const Tokenizer& t, const std::vector<std::string>& texts, int threads) {
        std::vector<std::vector<uint32_t>> out;
        { py::gil_scoped_release nogil; out = t.encode_batch(texts, threads); }
        py::list res;
        for (auto& v : out) res.append(to_array(v));
        return res;
      }, py::arg("texts"), py::arg("threads") = 0)
      .def("decode_bytes", [](const Tokenizer& t, py::handle ids) {
        return py::bytes(t.decode_bytes(ids_from(ids)));
      });

  py::class_<BpeTrainer>(m, "BpeTrainer")
      .def(py::init<>())
      .def("count", [](BpeTrainer& tr, const std::vector<std::string>& docs, int threads) {
        py::gil_scoped_release nogil;
        tr.count(docs, threads);
      }, py::arg("docs"), py::arg("threads") = 0)
      .def("train", [](BpeTrainer& tr, size_t n, int progress) {
        std::vector<std::string> merges;
        { py::gil_scoped_release nogil; merges = tr.train(n, progress); }
        py::list out;
        for (auto& s : merges) out.append(py::bytes(s));
        return out;
      }, py::arg("num_merges"), py::arg("progress") = 100)
      .def("unique_pretokens", &BpeTrainer::unique_pretokens);

  m.def("write_vocab", [](const std::string& path, const std::vector<py::bytes>& merges) {
    std::vector<std::string> ms;
    for (auto& b : merges) ms.emplace_back(std::string(b));
    write_vocab(path, ms);
  });

  py::class_<CropPacker>(m, "CropPacker")
      .def(py::init<int, int, int>(), py::arg("batch_rows"), py::arg("tokens_dim"), py::arg("buffer_size"))
      .def("push", [](CropPacker& p, py::handle ids) { p.push(ids_from(ids)); })
      .def("encode_and_push",
           [](CropPacker& p, const Tokenizer& tok, const std::vector<std::string>& texts, int threads) {
             // Tokenize documents, prepend BOS, drop ones that encode to nothing.
             std::vector<std::vector<uint32_t>> enc;
             {
               py::gil_scoped_release nogil;
               enc = tok.encode_batch(texts, threads);
             }
             size_t pushed = 0;
             for (auto& body : enc) {
               if (body.empty()) continue;
               std::vector<uint32_t> doc;
               doc.reserve(body.size() + 1);
               doc.push_back(tok.bos_id());
               doc.insert(doc.end(), body.begin(), body.end());
               p.push(std::move(doc));
               ++pushed;
             }
             return pushed;
           }, py::arg("tokenizer"), py::arg("texts"), py::arg("threads") = 0)
      .def("end_pass", &CropPacker::end_pass)
      .def("step", [](CropPacker& p) { py::gil_scoped_release nogil; return p.step(); })
      .def("take_rows", [](CropPacker& p) { return to_array(p.take_rows()); })
      .def("pending", &CropPacker::pending);

  py::class_<PackStats>(m, "PackStats")
      .def_readonly("rows", &PackStats::rows)
      .def_readonly("conversations", &PackStats::conversations)
      .def_readonly("pad_tokens", &PackStats::pad_tokens)
      .def_readonly("total_tokens", &PackStats::total_tokens)
      .def_readonly("scored_tokens", &PackStats::scored_tokens);

  py::class_<PackedEpoch>(m, "PackedEpoch")
      .def_property_readonly("rows", [](const PackedEpoch& e) { return to_array(e.rows); })
      .def_property_readonly("mask", [](const PackedEpoch& e) { return to_array(e.mask).attr("astype")("bool"); })
      .def_readonly("row_capacity", &PackedEpoch::row_capacity)
      .def_readonly("stats", &PackedEpoch::stats)
      .def("digest", &PackedEpoch::digest);

  m.def("pack_epoch", [](py::list rendered, size_t cap, uint32_t bos, size_t buffer_size) {
    std::vector<Rendered> rs;
    rs.reserve(rendered.size());
    for (py::handle h : rendered) {
      auto t = h.cast<py::tuple>();
      Rendered r;
      r.ids = ids_from(t[0]);
      auto mk = py::array_t<uint8_t, py::array::c_style | py::array::forcecast>::ensure(t[1]);
      r.mask.assign(mk.data(), mk.data() + mk.size());
      rs.push_back(std::move(r));
    }
    py::gil_scoped_release nogil;
    return pack_epoch(rs, cap, bos, buffer_size);
  }, py::arg("rendered"), py::arg("row_capacity"), py::arg("bos"), py::arg("buffer_size") = 100);

  m.def("render_conversation", [](const Tokenizer& tok, py::handle conv, size_t max_tokens) {
    return rendered_to_py(render_conversation(tok, conv_from(conv), max_tokens));
  });
  m.def("render_mixture", [](const Tokenizer& tok, py::list sources, const std::vector<std::string>& names,
                             size_t cap, uint64_t seed, int threads) {
    std::vector<std::vector<Conversation>> srcs;
    for (py::handle s : sources) {
      std::vector<Conversation> convs;
      for (py::handle c : s) convs.push_back(conv_from(c));
      srcs.push_back(std::move(convs));
    }
    std::vector<Rendered> out;
    {
      py::gil_scoped_release nogil;
      out = render_mixture(tok, srcs, names, cap, seed, threads);
    }
    py::list res;
    for (auto& r : out) res.append(rendered_to_py(r));
    return res;
  }, py::arg("tokenizer"), py::arg("sources"), py::arg("names"), py::arg("row_capacity"),
     py::arg("seed"), py::arg("threads") = 0);

  py::class_<ChaCha8>(m, "ChaCha8")
      .def(py::init<uint64_t>())
      .def("next_u32", &ChaCha8::next_u32)
      .def("next_u64", &ChaCha8::next_u64)
      .def("next_f64", &ChaCha8::next_f64)
      .def("shuffle_indices", [](ChaCha8& r, size_t n) {
        std::vector<uint32_t> idx(n);
        for (size_t i = 0; i < n; ++i) idx[i] = uint32_t(i);
        r.shuffle(n, [&](size_t i, size_t j) { std::swap(idx[i], idx[j]); });
        return to_array(idx);
      });
}
