// Composable launch programs: a model is a tree of modules whose forward enqueues kernels on the
// call's stream.
//
// Reference: the models crate composes typed modules (`Module` / `Op`, module.rs:8-35) with
// generic combinators (`Sequential`, `Fork`, `Layers`, `Choice`, ...; modules/generic/*) that its
// compiler schedules. Here the kernels are already fused, so a module is a short run of launches
// and the tree is built once per loaded model: a family is a different tree, tensor parallelism a
// different module at the same place, and the call's shape (decode rows, prompt chunks, kept rows)
// picks branches when the tree runs.
#pragma once

#include <functional>
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace foa::engine {

struct Launch;  // one call's launch state (model.cc): plan, stream, buffers, kernel accounting

class Module {
 public:
  virtual ~Module() = default;
  // Enqueues this module's kernels for the call described by `env`.
  virtual void forward(Launch& env) const = 0;
  // A short name for traces and for `describe`.
  virtual std::string name() const = 0;
  // The tree below this module, one line a module, indented by depth.
  virtual void describe(std::string& out, int depth) const {
    out += std::string(2 * depth, ' ') + name() + "\n";
  }
};

using ModulePtr = std::unique_ptr<Module>;

// Runs its parts in order.
class Sequential final : public Module {
 public:
  explicit Sequential(std::string name = "Sequential") : name_(std::move(name)) {}
  Sequential& then(ModulePtr m) {
    parts_.push_back(std::move(m));
    return *this;
  }
  void forward(Launch& env) const override {
    for (const auto& p : parts_) p->forward(env);
  }
  std::string name() const override { return name_; }
  void describe(std::string& out, int depth) const override {
    Module::describe(out, depth);
    for (const auto& p : parts_) p->describe(out, depth + 1);
  }
  size_t size() const { return parts_.size(); }

 private:
  std::string name_;
  std::vector<ModulePtr> parts_;
};

// `count` copies of a body built per layer index (unrolled: each layer holds its own weights).
class Layers final : public Module {
 public:
  Layers(int count, const std::function<ModulePtr(int)>& body) {
    for (int l = 0; l < count; ++l) layers_.push_back(body(l));
  }
  void forward(Launch& env) const override {
    for (const auto& l : layers_) l->forward(env);
  }
  std::string name() const override { return "Layers x" + std::to_string(layers_.size()); }
  void describe(std::string& out, int depth) const override {
    Module::describe(out, depth);
    if (!layers_.empty()) layers_.front()->describe(out, depth + 1);  // every layer has the same tree
  }

 private:
  std::vector<ModulePtr> layers_;
};

// One of two modules, picked per call by a predicate on the call (for example: the call has
// decode rows). A missing branch does nothing.
class Choice final : public Module {
 public:
  Choice(std::string name, std::function<bool(const Launch&)> pick, ModulePtr when_true, ModulePtr when_false = nullptr)
      : name_(std::move(name)), pick_(std::move(pick)), a_(std::move(when_true)), b_(std::move(when_false)) {}
  void forward(Launch& env) const override {
    const Module* m = pick_(env) ? a_.get() : b_.get();
    if (m != nullptr) m->forward(env);
  }
  std::string name() const override { return "Choice " + name_; }
  void describe(std::string& out, int depth) const override {
    Module::describe(out, depth);
    if (a_) a_->describe(out, depth + 1);
    if (b_) b_->describe(out, depth + 1);
  }

 private:
  std::string name_;
  std::function<bool(const Launch&)> pick_;
  ModulePtr a_, b_;
};

}  // namespace foa::engine
